"""Host-side decode step over the C ABI: the corrected counterpart of the KV
path of CacheFlow's BatchDecodeEngine::step (src/cacheflow/decode/
batch_decode.cpp:33-188).

The reference builds block tables, context lengths and slot mapping in host
memory (prepare_kv_cache_inputs, :92-131) and hands those host pointers, a
null query and a null output to the attention launcher (:137-176).  Here the
same host-side batch description is staged into device buffers owned by the
engine, the new K/V rows are scattered into the cache, attention runs on the
device, and the output is copied back -- all asynchronously on one stream.
The kernel choice follows the reference: v1 when the longest context is at
most 8192 tokens, else v2 with 512-token partitions (:162-177).
"""

from __future__ import annotations

import torch

from . import ops

V1_MAX_CONTEXT = 8192  # batch_decode.cpp:163


class DecodeEngine:
    def __init__(self, key_cache: torch.Tensor, value_cache: torch.Tensor, num_heads: int,
                 max_seqs: int, max_blocks_per_seq: int, max_new_tokens: int | None = None,
                 stream: torch.cuda.Stream | None = None, split_v1: bool = True):
        self.k = key_cache
        self.v = value_cache
        self.device = key_cache.device
        num_blocks, self.num_kv_heads, self.block_size, self.head_dim = key_cache.shape
        self.num_heads = num_heads
        self.max_seqs = max_seqs
        self.max_blocks_per_seq = max_blocks_per_seq
        self.max_new_tokens = max_new_tokens or max_seqs
        self.stream = stream or torch.cuda.current_stream(self.device)
        dt = key_cache.dtype
        dev = self.device
        self.q = torch.empty((max_seqs, num_heads, self.head_dim), dtype=dt, device=dev)
        self.out = torch.empty_like(self.q)
        self.k_new = torch.empty((self.max_new_tokens, self.num_kv_heads, self.head_dim), dtype=dt, device=dev)
        self.v_new = torch.empty_like(self.k_new)
        self.slots = torch.empty((self.max_new_tokens,), dtype=torch.int32, device=dev)
        self.tables = torch.empty((max_seqs, max_blocks_per_seq), dtype=torch.int32, device=dev)
        self.ctx = torch.empty((max_seqs,), dtype=torch.int32, device=dev)
        max_ctx = max_blocks_per_seq * self.block_size
        self.workspace = None
        if split_v1:
            n = ops.paged_attention_v1_workspace_size(self.q, key_cache, self.tables, min(max_ctx, V1_MAX_CONTEXT))
            if n:
                self.workspace = torch.empty((n,), dtype=torch.uint8, device=dev)
        self.parts = ops.v2_num_partitions(max_ctx)
        if max_ctx > V1_MAX_CONTEXT:
            self.exp_sums = torch.empty((max_seqs, num_heads, self.parts), dtype=torch.float32, device=dev)
            self.max_logits = torch.empty_like(self.exp_sums)
            self.tmp_out = torch.empty((max_seqs, num_heads, self.parts, self.head_dim), dtype=torch.float32,
                                       device=dev)
        self.launches_per_step = 0

    def h2d_bytes(self, num_seqs: int, num_new: int) -> int:
        e = self.q.element_size()
        return (num_seqs * self.num_heads * self.head_dim * e + 2 * num_new * self.num_kv_heads * self.head_dim * e
                + num_new * 4 + num_seqs * self.max_blocks_per_seq * 4 + num_seqs * 4)

    def d2h_bytes(self, num_seqs: int) -> int:
        return num_seqs * self.num_heads * self.head_dim * self.q.element_size()

    def attend(self, num_seqs: int, max_context_len: int) -> None:
        """Attention over device-resident inputs (q, tables, ctx already staged)."""
        S = num_seqs
        q, out, bt, cl = self.q[:S], self.out[:S], self.tables[:S], self.ctx[:S]
        if max_context_len <= V1_MAX_CONTEXT:
            ops.paged_attention_v1(out, q, self.k, self.v, bt, cl, None, max_context_len, workspace=self.workspace)
            self.launches_per_step = 1 + (1 if self.workspace is not None and max_context_len > 1024 else 0)
        else:
            P = self.parts
            ops.paged_attention_v2(out, self.exp_sums[:S], self.max_logits[:S], self.tmp_out[:S], q, self.k, self.v,
                                   bt, cl, None, max_context_len)
            self.launches_per_step = 2

    def step(self, q_host, k_new_host, v_new_host, slots_host, tables_host, ctx_host, out_host,
             max_context_len: int) -> None:
        """One decode step from pinned host buffers into pinned `out_host`.

        q_host [S, H, D]; k/v_new_host [T, Hkv, D]; slots_host int32 [T];
        tables_host int32 [S, max_blocks_per_seq]; ctx_host int32 [S].
        Asynchronous on the engine stream; synchronise before reading out_host.
        """
        S = q_host.shape[0]
        T = k_new_host.shape[0]
        with torch.cuda.stream(self.stream):
            self.q[:S].copy_(q_host, non_blocking=True)
            self.k_new[:T].copy_(k_new_host, non_blocking=True)
            self.v_new[:T].copy_(v_new_host, non_blocking=True)
            self.slots[:T].copy_(slots_host, non_blocking=True)
            self.tables[:S, : tables_host.shape[1]].copy_(tables_host, non_blocking=True)
            self.ctx[:S].copy_(ctx_host, non_blocking=True)
            ops.reshape_and_cache(self.k_new[:T], self.v_new[:T], self.k, self.v, self.slots[:T])
            self.attend(S, max_context_len)
            out_host.copy_(self.out[:S], non_blocking=True)
