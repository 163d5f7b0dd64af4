"""ctypes binding of libcacheflow_b200.so (the C ABI in include/cacheflow_b200.h).

This is the same binding any ctypes/cffi host would write; the library is
loaded from this package directory and nothing falls back to Python or CPU
code if it is missing.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int32, c_int64, c_size_t, c_uint8, c_uint32, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libcacheflow_b200.so")

# cf_status
CF_OK = 0
CF_ERR_INVALID_ARGUMENT = 1
CF_ERR_UNSUPPORTED = 2
CF_ERR_WORKSPACE = 3
CF_ERR_CUDA = 4
CF_ERR_PLAN = 5

# cf_dtype
CF_F32 = 0
CF_F16 = 1
CF_BF16 = 2
CF_FP8_E4M3 = 3

# device error bits
CF_DEVERR_BLOCK_ID = 0x1
CF_DEVERR_SLOT = 0x2
CF_DEVERR_CONTEXT_LEN = 0x4
CF_DEVERR_TIMEOUT = 0x8

CF_STATIC_SCRATCH_BYTES = 16 << 20


class AttentionParams(ctypes.Structure):
    """cf_paged_attention_params."""

    _fields_ = [
        ("query", c_void_p),
        ("key_cache", c_void_p),
        ("value_cache", c_void_p),
        ("output", c_void_p),
        ("block_tables", c_void_p),
        ("context_lens", c_void_p),
        ("scale", c_float),
        ("num_seqs", c_int32),
        ("num_heads", c_int32),
        ("num_kv_heads", c_int32),
        ("head_dim", c_int32),
        ("block_size", c_int32),
        ("max_context_len", c_int32),
        ("max_blocks_per_seq", c_int32),
        ("num_blocks", c_int64),
        ("dtype", c_int32),
    ]


class PrefillParams(ctypes.Structure):
    """cf_prefill_params."""

    _fields_ = [
        ("query", c_void_p),
        ("key_cache", c_void_p),
        ("value_cache", c_void_p),
        ("output", c_void_p),
        ("block_tables", c_void_p),
        ("context_lens", c_void_p),
        ("query_start", c_void_p),
        ("scale", c_float),
        ("num_chunks", c_int32),
        ("num_heads", c_int32),
        ("num_kv_heads", c_int32),
        ("head_dim", c_int32),
        ("block_size", c_int32),
        ("max_query_len", c_int32),
        ("max_blocks_per_seq", c_int32),
        ("num_blocks", c_int64),
        ("dtype", c_int32),
    ]


# name -> (restype, argtypes); exactly the functions include/cacheflow_b200.h declares.
SIGNATURES = {
    "cf_paged_attention_v1": (c_int32, [POINTER(AttentionParams), c_void_p, c_size_t, c_void_p]),
    "cf_paged_attention_v1_workspace_size": (c_size_t, [POINTER(AttentionParams)]),
    "cf_paged_attention_v2": (
        c_int32,
        [POINTER(AttentionParams), c_void_p, c_void_p, c_void_p, c_int32, c_void_p],
    ),
    "cf_paged_attention_v2_static_scratch": (c_int32, [POINTER(AttentionParams), c_void_p]),
    "cf_paged_attention_append_v1": (
        c_int32,
        [POINTER(AttentionParams), c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p],
    ),
    "cf_paged_attention_append_v2": (
        c_int32,
        [POINTER(AttentionParams), c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_int32, c_void_p],
    ),
    "cf_paged_attention_fp8_v1": (
        c_int32, [POINTER(AttentionParams), c_float, c_float, c_void_p, c_size_t, c_void_p],
    ),
    "cf_paged_attention_fp8_v2": (
        c_int32,
        [POINTER(AttentionParams), c_float, c_float, c_void_p, c_void_p, c_void_p, c_int32, c_void_p],
    ),
    "cf_paged_attention_fp8_append_v1": (
        c_int32,
        [POINTER(AttentionParams), c_float, c_float, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t,
         c_void_p],
    ),
    "cf_paged_attention_fp8_append_v2": (
        c_int32,
        [POINTER(AttentionParams), c_float, c_float, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p, c_int32, c_void_p],
    ),
    "cf_reshape_and_cache_fp8": (
        c_int32,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_int64,
         c_int32, c_float, c_float, c_void_p],
    ),
    "cf_build_decode_inputs": (
        c_int32,
        [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p,
         c_void_p],
    ),
    "cf_paged_prefill_attention": (c_int32, [POINTER(PrefillParams), c_void_p]),
    "cf_reshape_and_cache": (
        c_int32,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32,
         c_int64, c_int32, c_void_p],
    ),
    "cf_copy_blocks": (
        c_int32,
        [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_int64, c_int32,
         c_void_p],
    ),
    "cf_swap_blocks": (c_int32, [c_void_p, c_void_p, c_void_p, c_int32, c_int64, c_void_p]),
    "cf_swap_blocks_dma": (c_int32, [c_void_p, c_void_p, c_void_p, c_int32, c_int64, c_void_p]),
    "cf_execute_block_ops": (
        c_int32,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int32, c_void_p, c_int32,
         c_void_p, c_int32, c_void_p],
    ),
    "cf_compact_kv_cache": (
        c_int32,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_int64,
         c_int32, c_void_p],
    ),
    "cf_memset_blocks": (c_int32, [c_void_p, c_void_p, c_int32, c_int64, c_int64, c_void_p]),
    "cf_compaction_plan": (
        c_int32,
        [POINTER(c_uint8), c_int64, POINTER(c_int32), POINTER(c_int32), POINTER(c_int32)],
    ),
    "cf_check_compaction_plan": (c_int32, [POINTER(c_int32), POINTER(c_int32), c_int32, c_int64]),
    "cf_get_device_errors": (c_int32, [c_int32, POINTER(c_uint32), c_int32]),
    "cf_last_cuda_error": (c_int32, []),
    "cf_status_string": (c_char_p, [c_int32]),
    "cf_abi_version": (c_int32, []),
    "cf_testing_set_pipeline_faults": (c_int32, [c_int64, c_int32]),
}

# The C++ entry points with CacheFlow's signatures (mangled names).
COMPAT_SYMBOLS = [
    "cacheflow::cuda::launch_paged_attention_v1(cacheflow::cuda::PagedAttentionParams const&, CUstream_st*)",
    "cacheflow::cuda::launch_paged_attention_v2(cacheflow::cuda::PagedAttentionParams const&, float*, float*, float*, int, CUstream_st*)",
    "cacheflow::cuda::launch_reshape_and_cache(float const*, float const*, float*, float*, int const*, int, int, int, int, CUstream_st*)",
    "cacheflow::cuda::launch_copy_blocks(float*, float*, long const*, int, int, int, int, CUstream_st*)",
    "cacheflow::cuda::launch_swap_blocks(float*, float*, long const*, int, int, CUstream_st*)",
    "cacheflow::cuda::launch_compact_kv_cache(float*, float*, int const*, int const*, int, int, int, int, CUstream_st*)",
    "cacheflow::cuda::launch_memset_blocks(float*, int const*, int, int, CUstream_st*)",
    "cacheflow::cuda::get_gpu_free_memory()",
    "cacheflow::cuda::get_gpu_total_memory()",
    "cacheflow::cuda::get_gpu_memory_utilization()",
    "cacheflow::cuda::async_memcpy_h2d(void*, void const*, unsigned long, CUstream_st*)",
    "cacheflow::cuda::async_memcpy_d2h(void*, void const*, unsigned long, CUstream_st*)",
    "cacheflow::cuda::async_memcpy_d2d(void*, void const*, unsigned long, CUstream_st*)",
    "cacheflow::cuda::synchronize_stream(CUstream_st*)",
    "cacheflow::cuda::synchronize_device()",
]


class CacheFlowError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        msg = _LIB.cf_status_string(status).decode() if _LIB is not None else str(status)
        extra = ""
        if status == CF_ERR_CUDA and _LIB is not None:
            extra = f" (cudaError {_LIB.cf_last_cuda_error()})"
        super().__init__(f"{what}: {msg}{extra}")


_LIB: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Loads the library (once) and declares every C ABI signature."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m cacheflow_b200.build` "
            "(there is no fallback implementation)"
        )
    lib = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_LOCAL)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


def check(status: int, what: str) -> None:
    if status != CF_OK:
        raise CacheFlowError(status, what)
