"""PyTorch-facing operators over the C ABI.

One function per CacheFlow operator (src/cacheflow/cuda/*.cuh), same names and
argument meaning; tensors are CUDA tensors in CacheFlow's layouts:

    query / output   [num_seqs, num_heads, head_dim]
    key/value_cache  [num_blocks, num_kv_heads, block_size, head_dim]
    block_tables     int32 [num_seqs, max_blocks_per_seq]
    context_lens     int32 [num_seqs]

Every call is asynchronous on the current CUDA stream.  A non-OK status of the
library raises CacheFlowError; there is no fallback path.
"""

from __future__ import annotations

import ctypes
import math

import numpy as np
import torch

from . import _lib
from ._lib import AttentionParams, CacheFlowError, check

__all__ = [
    "CacheFlowError",
    "paged_attention_v1",
    "paged_attention_v1_workspace_size",
    "paged_attention_v2",
    "paged_prefill_attention",
    "paged_attention_append_v1",
    "paged_attention_append_v2",
    "paged_attention_fp8_v1",
    "paged_attention_fp8_v2",
    "reshape_and_cache_fp8",
    "build_decode_inputs",
    "v2_num_partitions",
    "reshape_and_cache",
    "copy_blocks",
    "swap_blocks",
    "swap_blocks_dma",
    "compact_kv_cache",
    "memset_blocks",
    "execute_block_ops",
    "compaction_plan",
    "check_compaction_plan",
    "device_errors",
    "dtype_code",
]

V2_PARTITION_TOKENS = 512

_DTYPES = {torch.float32: _lib.CF_F32, torch.float16: _lib.CF_F16, torch.bfloat16: _lib.CF_BF16,
           torch.float8_e4m3fn: _lib.CF_FP8_E4M3}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPES[dt]
    except KeyError:
        raise CacheFlowError(_lib.CF_ERR_UNSUPPORTED, f"dtype {dt}") from None


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _attention_params(out, query, key_cache, value_cache, block_tables, context_lens, scale,
                      max_context_len, fp8: bool = False) -> AttentionParams:
    for name, t in (("out", out), ("query", query), ("key_cache", key_cache),
                    ("value_cache", value_cache), ("block_tables", block_tables),
                    ("context_lens", context_lens)):
        if not t.is_contiguous():
            raise CacheFlowError(_lib.CF_ERR_INVALID_ARGUMENT, f"{name} must be contiguous")
    if block_tables.dtype != torch.int32 or context_lens.dtype != torch.int32:
        raise CacheFlowError(_lib.CF_ERR_INVALID_ARGUMENT, "block_tables/context_lens must be int32")
    if fp8:
        if not (key_cache.dtype == value_cache.dtype == torch.float8_e4m3fn and query.dtype == out.dtype):
            raise CacheFlowError(_lib.CF_ERR_INVALID_ARGUMENT,
                                 "fp8 attention: float8_e4m3fn caches, query and output of one 16-bit dtype")
    elif not (query.dtype == key_cache.dtype == value_cache.dtype == out.dtype):
        raise CacheFlowError(_lib.CF_ERR_INVALID_ARGUMENT, "query, caches and output must share a dtype")
    num_blocks, num_kv_heads, block_size, head_dim = key_cache.shape
    p = AttentionParams()
    p.query = _ptr(query)
    p.key_cache = _ptr(key_cache)
    p.value_cache = _ptr(value_cache)
    p.output = _ptr(out)
    p.block_tables = _ptr(block_tables)
    p.context_lens = _ptr(context_lens)
    p.scale = float(scale)
    p.num_seqs = query.shape[0]
    p.num_heads = query.shape[1]
    p.num_kv_heads = num_kv_heads
    p.head_dim = head_dim
    p.block_size = block_size
    p.max_context_len = int(max_context_len)
    p.max_blocks_per_seq = block_tables.shape[1] if block_tables.dim() == 2 else 0
    p.num_blocks = num_blocks
    p.dtype = dtype_code(query.dtype)
    return p


def paged_attention_v1_workspace_size(query, key_cache, block_tables, max_context_len) -> int:
    """Bytes of optional workspace that lets paged_attention_v1 split long contexts."""
    lib = _lib.load()
    p = AttentionParams()
    p.num_seqs = query.shape[0]
    p.num_heads = query.shape[1]
    _, p.num_kv_heads, p.block_size, p.head_dim = key_cache.shape
    p.max_context_len = int(max_context_len)
    p.max_blocks_per_seq = block_tables.shape[1]
    p.num_blocks = key_cache.shape[0]
    p.dtype = dtype_code(query.dtype)
    return int(lib.cf_paged_attention_v1_workspace_size(ctypes.byref(p)))


def paged_attention_v1(out, query, key_cache, value_cache, block_tables, context_lens, scale=None,
                       max_context_len=None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Decode attention (launch_paged_attention_v1, paged_attention.cuh:44-46)."""
    lib = _lib.load()
    if scale is None:
        scale = 1.0 / math.sqrt(query.shape[-1])
    if max_context_len is None:
        max_context_len = int(context_lens.max().item()) if context_lens.numel() else 0
    p = _attention_params(out, query, key_cache, value_cache, block_tables, context_lens, scale,
                          max_context_len)
    ws = _ptr(workspace)
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    check(lib.cf_paged_attention_v1(ctypes.byref(p), ws, ws_bytes, _stream(query)),
          "cf_paged_attention_v1")
    return out


def v2_num_partitions(max_context_len: int) -> int:
    return max(1, (int(max_context_len) + V2_PARTITION_TOKENS - 1) // V2_PARTITION_TOKENS)


def paged_attention_v2(out, exp_sums, max_logits, tmp_output, query, key_cache, value_cache,
                       block_tables, context_lens, scale=None, max_context_len=None) -> torch.Tensor:
    """Partitioned decode attention + reduce (launch_paged_attention_v2, paged_attention.cuh:48-54).

    exp_sums / max_logits: float32 [num_seqs, num_heads, P];
    tmp_output: float32 [num_seqs, num_heads, P, head_dim]; P >= v2_num_partitions(max_context_len).
    """
    lib = _lib.load()
    if scale is None:
        scale = 1.0 / math.sqrt(query.shape[-1])
    if max_context_len is None:
        max_context_len = int(context_lens.max().item()) if context_lens.numel() else 0
    p = _attention_params(out, query, key_cache, value_cache, block_tables, context_lens, scale,
                          max_context_len)
    for t in (exp_sums, max_logits, tmp_output):
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise CacheFlowError(_lib.CF_ERR_INVALID_ARGUMENT, "v2 scratch must be contiguous float32")
    parts = exp_sums.shape[-1]
    check(lib.cf_paged_attention_v2(ctypes.byref(p), _ptr(exp_sums), _ptr(max_logits),
                                    _ptr(tmp_output), parts, _stream(query)),
          "cf_paged_attention_v2")
    return out


def _check_new_rows(key, value, query, key_cache):
    want = (query.shape[0], key_cache.shape[1], key_cache.shape[3])
    dt = query.dtype if key_cache.dtype == torch.float8_e4m3fn else key_cache.dtype
    for name, t in (("key", key), ("value", value)):
        if tuple(t.shape) != want or t.dtype != dt or not t.is_contiguous():
            raise CacheFlowError(_lib.CF_ERR_INVALID_ARGUMENT,
                                 f"{name} must be contiguous {dt} of shape {want}")


def paged_attention_append_v1(out, query, key, value, key_cache, value_cache, block_tables, context_lens,
                              slot_mapping=None, scale=None, max_context_len=None,
                              workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Fused decode step: reshape_and_cache of every row's newest token (at
    position context_lens[s] - 1) followed by paged_attention_v1, in one launch.

    key/value: [num_seqs, num_kv_heads, head_dim]; slot_mapping: int32 [num_seqs]
    or None (the slot comes from the block table).  Writes key_cache/value_cache.
    """
    lib = _lib.load()
    _check_new_rows(key, value, query, key_cache)
    if scale is None:
        scale = 1.0 / math.sqrt(query.shape[-1])
    if max_context_len is None:
        max_context_len = int(context_lens.max().item()) if context_lens.numel() else 0
    p = _attention_params(out, query, key_cache, value_cache, block_tables, context_lens, scale,
                          max_context_len)
    ws = _ptr(workspace)
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    check(lib.cf_paged_attention_append_v1(ctypes.byref(p), _ptr(key), _ptr(value), _ptr(slot_mapping),
                                           ws, ws_bytes, _stream(query)),
          "cf_paged_attention_append_v1")
    return out


def paged_attention_append_v2(out, exp_sums, max_logits, tmp_output, query, key, value, key_cache,
                              value_cache, block_tables, context_lens, slot_mapping=None, scale=None,
                              max_context_len=None) -> torch.Tensor:
    """Fused decode step on the partitioned path: reshape_and_cache of every
    row's newest token followed by paged_attention_v2, in one partition launch
    (+ the reduce)."""
    lib = _lib.load()
    _check_new_rows(key, value, query, key_cache)
    if scale is None:
        scale = 1.0 / math.sqrt(query.shape[-1])
    if max_context_len is None:
        max_context_len = int(context_lens.max().item()) if context_lens.numel() else 0
    p = _attention_params(out, query, key_cache, value_cache, block_tables, context_lens, scale,
                          max_context_len)
    for t in (exp_sums, max_logits, tmp_output):
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise CacheFlowError(_lib.CF_ERR_INVALID_ARGUMENT, "v2 scratch must be contiguous float32")
    check(lib.cf_paged_attention_append_v2(ctypes.byref(p), _ptr(key), _ptr(value), _ptr(slot_mapping),
                                           _ptr(exp_sums), _ptr(max_logits), _ptr(tmp_output),
                                           exp_sums.shape[-1], _stream(query)),
          "cf_paged_attention_append_v2")
    return out


def paged_attention_fp8_v1(out, query, key_cache, value_cache, block_tables, context_lens, k_scale, v_scale,
                           scale=None, max_context_len=None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Decode attention over float8_e4m3fn caches holding K / k_scale and V / v_scale
    (query and output f16 or bf16); workspace as paged_attention_v1."""
    lib = _lib.load()
    if scale is None:
        scale = 1.0 / math.sqrt(query.shape[-1])
    if max_context_len is None:
        max_context_len = int(context_lens.max().item()) if context_lens.numel() else 0
    p = _attention_params(out, query, key_cache, value_cache, block_tables, context_lens, scale,
                          max_context_len, fp8=True)
    ws = _ptr(workspace)
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    check(lib.cf_paged_attention_fp8_v1(ctypes.byref(p), float(k_scale), float(v_scale), ws, ws_bytes,
                                        _stream(query)),
          "cf_paged_attention_fp8_v1")
    return out


def paged_attention_fp8_v2(out, exp_sums, max_logits, tmp_output, query, key_cache, value_cache, block_tables,
                           context_lens, k_scale, v_scale, scale=None, max_context_len=None) -> torch.Tensor:
    """Partitioned form of paged_attention_fp8_v1 (scratch as paged_attention_v2)."""
    lib = _lib.load()
    if scale is None:
        scale = 1.0 / math.sqrt(query.shape[-1])
    if max_context_len is None:
        max_context_len = int(context_lens.max().item()) if context_lens.numel() else 0
    p = _attention_params(out, query, key_cache, value_cache, block_tables, context_lens, scale,
                          max_context_len, fp8=True)
    for t in (exp_sums, max_logits, tmp_output):
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise CacheFlowError(_lib.CF_ERR_INVALID_ARGUMENT, "v2 scratch must be contiguous float32")
    check(lib.cf_paged_attention_fp8_v2(ctypes.byref(p), float(k_scale), float(v_scale), _ptr(exp_sums),
                                        _ptr(max_logits), _ptr(tmp_output), exp_sums.shape[-1], _stream(query)),
          "cf_paged_attention_fp8_v2")
    return out


def paged_attention_fp8_append_v1(out, query, key, value, key_cache, value_cache, block_tables, context_lens,
                                  k_scale, v_scale, slot_mapping=None, scale=None, max_context_len=None,
                                  workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Fused decode step over float8_e4m3fn caches: reshape_and_cache_fp8 of
    every row's newest token (key/value of the query dtype) followed by
    paged_attention_fp8_v1, in one launch (rules as paged_attention_append_v1)."""
    lib = _lib.load()
    _check_new_rows(key, value, query, key_cache)
    if scale is None:
        scale = 1.0 / math.sqrt(query.shape[-1])
    if max_context_len is None:
        max_context_len = int(context_lens.max().item()) if context_lens.numel() else 0
    p = _attention_params(out, query, key_cache, value_cache, block_tables, context_lens, scale,
                          max_context_len, fp8=True)
    ws = _ptr(workspace)
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    check(lib.cf_paged_attention_fp8_append_v1(ctypes.byref(p), float(k_scale), float(v_scale), _ptr(key),
                                               _ptr(value), _ptr(slot_mapping), ws, ws_bytes, _stream(query)),
          "cf_paged_attention_fp8_append_v1")
    return out


def paged_attention_fp8_append_v2(out, exp_sums, max_logits, tmp_output, query, key, value, key_cache,
                                  value_cache, block_tables, context_lens, k_scale, v_scale, slot_mapping=None,
                                  scale=None, max_context_len=None) -> torch.Tensor:
    """Partitioned form of paged_attention_fp8_append_v1 (scratch as paged_attention_v2)."""
    lib = _lib.load()
    _check_new_rows(key, value, query, key_cache)
    if scale is None:
        scale = 1.0 / math.sqrt(query.shape[-1])
    if max_context_len is None:
        max_context_len = int(context_lens.max().item()) if context_lens.numel() else 0
    p = _attention_params(out, query, key_cache, value_cache, block_tables, context_lens, scale,
                          max_context_len, fp8=True)
    for t in (exp_sums, max_logits, tmp_output):
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise CacheFlowError(_lib.CF_ERR_INVALID_ARGUMENT, "v2 scratch must be contiguous float32")
    check(lib.cf_paged_attention_fp8_append_v2(ctypes.byref(p), float(k_scale), float(v_scale), _ptr(key),
                                               _ptr(value), _ptr(slot_mapping), _ptr(exp_sums),
                                               _ptr(max_logits), _ptr(tmp_output), exp_sums.shape[-1],
                                               _stream(query)),
          "cf_paged_attention_fp8_append_v2")
    return out


def reshape_and_cache_fp8(key, value, key_cache, value_cache, slot_mapping, k_scale, v_scale) -> None:
    """reshape_and_cache into float8_e4m3fn caches: cache = e4m3(x / scale)."""
    lib = _lib.load()
    num_blocks, num_kv_heads, block_size, head_dim = key_cache.shape
    if slot_mapping.dtype != torch.int32:
        raise CacheFlowError(_lib.CF_ERR_INVALID_ARGUMENT, "slot_mapping must be int32")
    if key_cache.dtype != torch.float8_e4m3fn or value_cache.dtype != torch.float8_e4m3fn:
        raise CacheFlowError(_lib.CF_ERR_INVALID_ARGUMENT, "caches must be float8_e4m3fn")
    if not (key.is_contiguous() and value.is_contiguous() and key.dtype == value.dtype):
        raise CacheFlowError(_lib.CF_ERR_INVALID_ARGUMENT, "key/value must be contiguous, of one dtype")
    check(lib.cf_reshape_and_cache_fp8(_ptr(key), _ptr(value), _ptr(key_cache), _ptr(value_cache),
                                       _ptr(slot_mapping), key.shape[0], num_kv_heads, head_dim, block_size,
                                       num_blocks, dtype_code(key.dtype), float(k_scale), float(v_scale),
                                       _stream(key_cache)),
          "cf_reshape_and_cache_fp8")


def build_decode_inputs(positions, block_offsets, block_ids, max_blocks_per_seq, block_size=16,
                        block_tables=None, context_lens=None, slot_mapping=None):
    """Device-side prepare_kv_cache_inputs (batch_decode.cpp:92-131).

    positions: int32 [S]; block_offsets: int64 [S + 1]; block_ids: int32 (row s
    owns block_ids[block_offsets[s]:block_offsets[s + 1]]).  Returns
    (block_tables int32 [S, max_blocks_per_seq], context_lens int32 [S],
    slot_mapping int32 [S]), allocated when not given.
    """
    lib = _lib.load()
    S = positions.shape[0]
    dev = positions.device
    for name, t, dt in (("positions", positions, torch.int32), ("block_offsets", block_offsets, torch.int64),
                        ("block_ids", block_ids, torch.int32)):
        if t.dtype != dt or not t.is_contiguous() or t.device != dev:
            raise CacheFlowError(_lib.CF_ERR_INVALID_ARGUMENT, f"{name} must be contiguous {dt} on {dev}")
    if block_offsets.shape[0] != S + 1:
        raise CacheFlowError(_lib.CF_ERR_INVALID_ARGUMENT, "block_offsets must have num_seqs + 1 entries")
    if block_tables is None:
        block_tables = torch.empty((S, max_blocks_per_seq), dtype=torch.int32, device=dev)
    if context_lens is None:
        context_lens = torch.empty((S,), dtype=torch.int32, device=dev)
    if slot_mapping is None:
        slot_mapping = torch.empty((S,), dtype=torch.int32, device=dev)
    if block_ids.numel() == 0:
        block_ids = torch.zeros((1,), dtype=torch.int32, device=dev)
    check(lib.cf_build_decode_inputs(_ptr(positions), _ptr(block_offsets), _ptr(block_ids), S,
                                     int(max_blocks_per_seq), int(block_size), _ptr(block_tables),
                                     _ptr(context_lens), _ptr(slot_mapping), _stream(positions)),
          "cf_build_decode_inputs")
    return block_tables, context_lens, slot_mapping


def paged_prefill_attention(out, query, key_cache, value_cache, block_tables, context_lens, query_start,
                            scale=None, max_query_len=None) -> torch.Tensor:
    """Chunked-prefill attention (no CacheFlow counterpart).

    query/out: [total query tokens, num_heads, head_dim]; block_tables int32
    [num_chunks, max_blocks_per_seq]; context_lens int32 [num_chunks] (the
    chunk's tokens included, already in the cache); query_start int32
    [num_chunks + 1].  Query token i of chunk c sits at position
    context_lens[c] - n_c + i and attends causally.
    """
    lib = _lib.load()
    if scale is None:
        scale = 1.0 / math.sqrt(query.shape[-1])
    if max_query_len is None:
        max_query_len = int((query_start[1:] - query_start[:-1]).max().item()) if query_start.numel() > 1 else 0
    for name, t in (("out", out), ("query", query), ("key_cache", key_cache), ("value_cache", value_cache),
                    ("block_tables", block_tables), ("context_lens", context_lens), ("query_start", query_start)):
        if not t.is_contiguous():
            raise CacheFlowError(_lib.CF_ERR_INVALID_ARGUMENT, f"{name} must be contiguous")
    num_blocks, num_kv_heads, block_size, head_dim = key_cache.shape
    p = _lib.PrefillParams()
    p.query, p.key_cache, p.value_cache, p.output = _ptr(query), _ptr(key_cache), _ptr(value_cache), _ptr(out)
    p.block_tables, p.context_lens, p.query_start = _ptr(block_tables), _ptr(context_lens), _ptr(query_start)
    p.scale = float(scale)
    p.num_chunks = context_lens.shape[0]
    p.num_heads = query.shape[1]
    p.num_kv_heads = num_kv_heads
    p.head_dim = head_dim
    p.block_size = block_size
    p.max_query_len = int(max_query_len)
    p.max_blocks_per_seq = block_tables.shape[1]
    p.num_blocks = num_blocks
    p.dtype = dtype_code(query.dtype)
    check(lib.cf_paged_prefill_attention(ctypes.byref(p), _stream(query)), "cf_paged_prefill_attention")
    return out


def reshape_and_cache(key, value, key_cache, value_cache, slot_mapping) -> None:
    """Scatter new K/V rows into their slots (launch_reshape_and_cache, kv_cache_kernels.cuh:17-27)."""
    lib = _lib.load()
    num_blocks, num_kv_heads, block_size, head_dim = key_cache.shape
    if slot_mapping.dtype != torch.int32:
        raise CacheFlowError(_lib.CF_ERR_INVALID_ARGUMENT, "slot_mapping must be int32")
    check(lib.cf_reshape_and_cache(_ptr(key), _ptr(value), _ptr(key_cache), _ptr(value_cache),
                                   _ptr(slot_mapping), key.shape[0], num_kv_heads, head_dim,
                                   block_size, num_blocks, dtype_code(key_cache.dtype),
                                   _stream(key_cache)),
          "cf_reshape_and_cache")


def copy_blocks(key_cache, value_cache, block_mapping) -> None:
    """COW block copies (launch_copy_blocks, kv_cache_kernels.cuh:29-37); block_mapping int64 [N, 2]."""
    lib = _lib.load()
    num_blocks, num_kv_heads, block_size, head_dim = key_cache.shape
    if block_mapping.dtype != torch.int64:
        raise CacheFlowError(_lib.CF_ERR_INVALID_ARGUMENT, "block_mapping must be int64")
    check(lib.cf_copy_blocks(_ptr(key_cache), _ptr(value_cache), _ptr(block_mapping),
                             block_mapping.shape[0], num_kv_heads, head_dim, block_size,
                             num_blocks, dtype_code(key_cache.dtype), _stream(key_cache)),
          "cf_copy_blocks")


def _block_bytes(cache: torch.Tensor) -> int:
    return cache[0].numel() * cache.element_size()


def swap_blocks(src, dst, block_mapping, stream_tensor: torch.Tensor | None = None) -> None:
    """SM-driven block copy between caches (launch_swap_blocks, kv_cache_kernels.cuh:39-45).

    One of src/dst may be pinned host memory; block_mapping int64 [N, 2] must be
    device-readable (a CUDA tensor or pinned host tensor).
    """
    lib = _lib.load()
    dev_t = stream_tensor if stream_tensor is not None else (src if src.is_cuda else dst)
    check(lib.cf_swap_blocks(_ptr(src), _ptr(dst), _ptr(block_mapping), block_mapping.shape[0],
                             _block_bytes(src), _stream(dev_t)),
          "cf_swap_blocks")


def swap_blocks_dma(src, dst, block_mapping_host: np.ndarray | torch.Tensor,
                    stream_tensor: torch.Tensor | None = None) -> None:
    """Copy-engine swap: block_mapping in host memory, consecutive runs merged."""
    lib = _lib.load()
    m = block_mapping_host
    if isinstance(m, torch.Tensor):
        m = m.cpu().numpy()
    m = np.ascontiguousarray(m, dtype=np.int64)
    dev_t = stream_tensor if stream_tensor is not None else (src if src.is_cuda else dst)
    check(lib.cf_swap_blocks_dma(_ptr(src), _ptr(dst), m.ctypes.data, m.shape[0], _block_bytes(src),
                                 _stream(dev_t)),
          "cf_swap_blocks_dma")


def compact_kv_cache(key_cache, value_cache, src_block_ids, dst_block_ids) -> None:
    """In-place defragmentation moves (launch_compact_kv_cache, kv_cache_kernels.cuh:47-56)."""
    lib = _lib.load()
    num_blocks, num_kv_heads, block_size, head_dim = key_cache.shape
    if src_block_ids.dtype != torch.int32 or dst_block_ids.dtype != torch.int32:
        raise CacheFlowError(_lib.CF_ERR_INVALID_ARGUMENT, "block ids must be int32")
    check(lib.cf_compact_kv_cache(_ptr(key_cache), _ptr(value_cache), _ptr(src_block_ids),
                                  _ptr(dst_block_ids), src_block_ids.shape[0], num_kv_heads,
                                  head_dim, block_size, num_blocks, dtype_code(key_cache.dtype),
                                  _stream(key_cache)),
          "cf_compact_kv_cache")


def memset_blocks(cache, block_ids) -> None:
    """Zero listed blocks (launch_memset_blocks, memory_utils.cuh:28-33)."""
    lib = _lib.load()
    check(lib.cf_memset_blocks(_ptr(cache), _ptr(block_ids), block_ids.shape[0], _block_bytes(cache),
                               cache.shape[0], _stream(cache)),
          "cf_memset_blocks")


def execute_block_ops(gpu_key_cache, gpu_value_cache, cpu_key_cache, cpu_value_cache, swaps_out=None,
                      swaps_in=None, copies=None) -> None:
    """One scheduling step's block operations (SchedulerOutput::block_swaps_out,
    block_swaps_in, block_copies): swap-outs, swap-ins, then copy-on-write
    copies, for K and V.  Pair lists are host int64 arrays [n, 2] of (src, dst)
    block ids; scattered lists run on the SM copy kernel, lists of long
    contiguous runs (and pageable CPU pools) on the copy engines."""
    lib = _lib.load()

    def host_pairs(x):
        if x is None:
            return None, 0
        a = np.ascontiguousarray(np.asarray(x, dtype=np.int64).reshape(-1, 2))
        return a, a.shape[0]

    so, nso = host_pairs(swaps_out)
    si, nsi = host_pairs(swaps_in)
    cp, ncp = host_pairs(copies)
    cpu_k = _ptr(cpu_key_cache) if cpu_key_cache is not None else None
    cpu_v = _ptr(cpu_value_cache) if cpu_value_cache is not None else None
    ncpu = cpu_key_cache.shape[0] if cpu_key_cache is not None else 0
    check(lib.cf_execute_block_ops(_ptr(gpu_key_cache), _ptr(gpu_value_cache), cpu_k, cpu_v,
                                   _block_bytes(gpu_key_cache), gpu_key_cache.shape[0], ncpu,
                                   None if so is None else so.ctypes.data, nso,
                                   None if si is None else si.ctypes.data, nsi,
                                   None if cp is None else cp.ctypes.data, ncp, _stream(gpu_key_cache)),
          "cf_execute_block_ops")


def compaction_plan(used: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Host planner: moves that pack live blocks below num_used without overlap."""
    lib = _lib.load()
    u = np.ascontiguousarray(used, dtype=np.uint8)
    n = u.shape[0]
    src = np.empty(max(n, 1), dtype=np.int32)
    dst = np.empty(max(n, 1), dtype=np.int32)
    cnt = ctypes.c_int32(0)
    check(lib.cf_compaction_plan(u.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), n,
                                 src.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                 dst.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                 ctypes.byref(cnt)),
          "cf_compaction_plan")
    return src[: cnt.value].copy(), dst[: cnt.value].copy()


def check_compaction_plan(src: np.ndarray, dst: np.ndarray, num_blocks: int) -> int:
    """Returns the cf_status of the host-side race check (CF_OK, CF_ERR_PLAN, ...)."""
    lib = _lib.load()
    s = np.ascontiguousarray(src, dtype=np.int32)
    d = np.ascontiguousarray(dst, dtype=np.int32)
    return int(lib.cf_check_compaction_plan(s.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                            d.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                            s.shape[0], int(num_blocks)))


def device_errors(device: int = 0, clear: bool = True) -> int:
    """OR of CF_DEVERR_* bits recorded by kernels on `device` (synchronises it)."""
    lib = _lib.load()
    bits = ctypes.c_uint32(0)
    check(lib.cf_get_device_errors(int(device), ctypes.byref(bits), 1 if clear else 0),
          "cf_get_device_errors")
    return int(bits.value)
