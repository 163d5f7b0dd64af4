"""Host-side decode step over the C ABI: the corrected counterpart of the KV
path of CacheFlow's BatchDecodeEngine::step (src/cacheflow/decode/
batch_decode.cpp:33-188).

The reference builds block tables, context lengths and slot mapping in host
memory (prepare_kv_cache_inputs, :92-131) and hands those host pointers, a
null query and a null output to the attention launcher (:137-176).  Here the
same host-side batch description is staged into device buffers owned by the
engine, the new K/V rows are scattered into the cache, attention runs on the
device, and the output is copied back.  Attention runs v1 with the
library's own context split for every length (kernel="v1", the default:
4096- or 8192-token partitions past 8192 tokens write an eighth or less of
v2's partial results), or follows the reference's choice (kernel="reference": v1 when the
longest context is at most 8192 tokens, else v2 with 512-token partitions,
:162-177).

Steps are pipelined over `depth` staging slots and three streams: the
host-to-device copies of step i+1 and the device-to-host copy of step i-1
run on the copy engines while step i computes.  Every dependency is an event:
a slot's inputs are overwritten only after the step that read them finished,
its output only after it was copied out.
"""

from __future__ import annotations

import torch

from . import ops

V1_MAX_CONTEXT = 8192  # batch_decode.cpp:163


class _Slot:
    def __init__(self, max_seqs, max_new, num_heads, num_kv_heads, head_dim, max_blocks, dt, dev, max_chunks):
        self.q = torch.empty((max_seqs, num_heads, head_dim), dtype=dt, device=dev)
        self.out = torch.empty_like(self.q)
        self.k_new = torch.empty((max_new, num_kv_heads, head_dim), dtype=dt, device=dev)
        self.v_new = torch.empty_like(self.k_new)
        self.slots = torch.empty((max_new,), dtype=torch.int32, device=dev)
        self.tables = torch.empty((max_seqs, max_blocks), dtype=torch.int32, device=dev)
        self.ctx = torch.empty((max_seqs,), dtype=torch.int32, device=dev)
        self.c_tables = torch.empty((max_chunks, max_blocks), dtype=torch.int32, device=dev)
        self.c_ctx = torch.empty((max_chunks,), dtype=torch.int32, device=dev)
        self.c_start = torch.empty((max_chunks + 1,), dtype=torch.int32, device=dev)
        self.h2d_done = torch.cuda.Event()
        self.compute_done = torch.cuda.Event()
        self.d2h_done = torch.cuda.Event()
        self.used = False


class DecodeEngine:
    def __init__(self, key_cache: torch.Tensor, value_cache: torch.Tensor, num_heads: int,
                 max_seqs: int, max_blocks_per_seq: int, max_new_tokens: int | None = None,
                 stream: torch.cuda.Stream | None = None, split_v1: bool = True, depth: int = 2,
                 max_chunks: int = 0, fused_append: bool = False, kv_scales: tuple[float, float] | None = None,
                 query_dtype: torch.dtype | None = None, kernel: str = "v1"):
        """kv_scales = (k_scale, v_scale) with float8_e4m3fn caches: the caches
        hold K / k_scale and V / v_scale; queries, new K/V rows and outputs are
        `query_dtype` (f16 / bf16).  kernel = "v1" (v1 with the library's
        split at every context length) or "reference" (v1 up to 8192 tokens,
        v2 beyond, as CacheFlow's engine chooses)."""
        if kernel not in ("v1", "reference"):
            raise ValueError("kernel must be 'v1' or 'reference'")
        self.k = key_cache
        self.v = value_cache
        self.device = key_cache.device
        _, self.num_kv_heads, self.block_size, self.head_dim = key_cache.shape
        self.num_heads = num_heads
        self.max_seqs = max_seqs
        self.max_blocks_per_seq = max_blocks_per_seq
        self.max_new_tokens = max_new_tokens or max_seqs
        self.stream = stream or torch.cuda.current_stream(self.device)
        self.h2d = torch.cuda.Stream(self.device)
        self.d2h = torch.cuda.Stream(self.device)
        self.fp8 = key_cache.dtype == torch.float8_e4m3fn
        if self.fp8 and (kv_scales is None or query_dtype is None):
            raise ValueError("fp8 caches need kv_scales and query_dtype")
        self.kv_scales = kv_scales
        dt, dev = (query_dtype if self.fp8 else key_cache.dtype), self.device
        self.slots_ = [_Slot(max_seqs, self.max_new_tokens, num_heads, self.num_kv_heads, self.head_dim,
                             max_blocks_per_seq, dt, dev, max_chunks) for _ in range(max(1, depth))]
        self.c_tables, self.c_ctx, self.c_start = self.slots_[0].c_tables, self.slots_[0].c_ctx, self.slots_[0].c_start
        self.n = 0
        # slot 0 doubles as the buffer set of attend() for device-resident inputs
        s0 = self.slots_[0]
        self.q, self.out, self.tables, self.ctx = s0.q, s0.out, s0.tables, s0.ctx
        max_ctx = max_blocks_per_seq * self.block_size
        # contexts longer than this run v2 (None: never)
        self.v2_above = V1_MAX_CONTEXT if kernel == "reference" else None
        self.workspace = None
        if split_v1:
            v1_ctx = max_ctx if self.v2_above is None else min(max_ctx, self.v2_above)
            n = ops.paged_attention_v1_workspace_size(self.q, key_cache, self.tables, v1_ctx)
            if n:
                self.workspace = torch.empty((n,), dtype=torch.uint8, device=dev)
        self.parts = ops.v2_num_partitions(max_ctx)
        if self.v2_above is not None and max_ctx > self.v2_above:
            self.exp_sums = torch.empty((max_seqs, num_heads, self.parts), dtype=torch.float32, device=dev)
            self.max_logits = torch.empty_like(self.exp_sums)
            self.tmp_out = torch.empty((max_seqs, num_heads, self.parts, self.head_dim), dtype=torch.float32,
                                       device=dev)
        self.launches_per_step = 0
        self.side = None  # created by the first mixed step
        # Decode steps whose new tokens are exactly one per row, at each row's
        # newest position, append and attend in one launch
        # (paged_attention_append_v1/_v2) instead of reshape_and_cache + attention.
        self.fused_append = fused_append

    def h2d_bytes(self, num_seqs: int, num_new: int) -> int:
        e = self.q.element_size()
        return (num_seqs * self.num_heads * self.head_dim * e + 2 * num_new * self.num_kv_heads * self.head_dim * e
                + num_new * 4 + num_seqs * self.max_blocks_per_seq * 4 + num_seqs * 4)

    def d2h_bytes(self, num_seqs: int) -> int:
        return num_seqs * self.num_heads * self.head_dim * self.q.element_size()

    def _use_v2(self, max_context_len: int) -> bool:
        return self.v2_above is not None and max_context_len > self.v2_above

    def _attend(self, q, out, bt, cl, num_seqs: int, max_context_len: int, new=None) -> None:
        """new = (k_new, v_new, slot_mapping) of one token per row appends it
        in the same launch."""
        S = num_seqs
        if self.fp8:
            ks, vs = self.kv_scales
            fused = new is not None and self.fused_append
            if new is not None and not fused:
                ops.reshape_and_cache_fp8(new[0], new[1], self.k, self.v, new[2], ks, vs)
            extra = 1 if new is not None and not fused else 0
            if not self._use_v2(max_context_len):
                if fused:
                    ops.paged_attention_fp8_append_v1(out, q, new[0], new[1], self.k, self.v, bt, cl, ks, vs, new[2],
                                                      None, max_context_len, workspace=self.workspace)
                else:
                    ops.paged_attention_fp8_v1(out, q, self.k, self.v, bt, cl, ks, vs, None, max_context_len,
                                               workspace=self.workspace)
                split = self.workspace is not None and ops.paged_attention_v1_workspace_size(
                    q, self.k, bt, max_context_len) > 0
                self.launches_per_step = (2 if split else 1) + extra
            else:
                if fused:
                    ops.paged_attention_fp8_append_v2(out, self.exp_sums[:S], self.max_logits[:S], self.tmp_out[:S],
                                                      q, new[0], new[1], self.k, self.v, bt, cl, ks, vs, new[2],
                                                      None, max_context_len)
                else:
                    ops.paged_attention_fp8_v2(out, self.exp_sums[:S], self.max_logits[:S], self.tmp_out[:S], q,
                                               self.k, self.v, bt, cl, ks, vs, None, max_context_len)
                self.launches_per_step = 2 + extra
            return
        if not self._use_v2(max_context_len):
            if new is None:
                ops.paged_attention_v1(out, q, self.k, self.v, bt, cl, None, max_context_len,
                                       workspace=self.workspace)
            else:
                ops.paged_attention_append_v1(out, q, new[0], new[1], self.k, self.v, bt, cl, new[2], None,
                                              max_context_len, workspace=self.workspace)
            split = self.workspace is not None and ops.paged_attention_v1_workspace_size(
                q, self.k, bt, max_context_len) > 0
            self.launches_per_step = 2 if split else 1
        else:
            if new is None:
                ops.paged_attention_v2(out, self.exp_sums[:S], self.max_logits[:S], self.tmp_out[:S], q, self.k,
                                       self.v, bt, cl, None, max_context_len)
            else:
                ops.paged_attention_append_v2(out, self.exp_sums[:S], self.max_logits[:S], self.tmp_out[:S], q,
                                              new[0], new[1], self.k, self.v, bt, cl, new[2], None,
                                              max_context_len)
            self.launches_per_step = 2

    def _attend_mixed(self, b, num_seqs, max_context_len, chunks):
        """Decode rows [0, num_decode) with paged attention, the remaining rows
        as prefill chunks with the multi-query operator.  The two launches run
        concurrently: the prefill (tensor-bound) on the current stream, the
        decode rows (HBM-bound) on a high-priority side stream forked from it
        and joined back into it, so the decode CTAs take SMs as the prefill's
        retire instead of waiting for the whole prefill grid."""
        nd, nc, max_q = chunks
        cur = torch.cuda.current_stream(self.device)
        if nd:
            if self.side is None:
                self.side = torch.cuda.Stream(self.device, priority=-5)  # clamped to the highest
                self.fork, self.joined = torch.cuda.Event(), torch.cuda.Event()
            self.fork.record(cur)
            self.side.wait_event(self.fork)
        ops.paged_prefill_attention(b.out[nd:num_seqs], b.q[nd:num_seqs], self.k, self.v, b.c_tables[:nc],
                                    b.c_ctx[:nc], b.c_start[: nc + 1], None, max_q)
        if nd:
            with torch.cuda.stream(self.side):
                self._attend(b.q[:nd], b.out[:nd], b.tables[:nd], b.ctx[:nd], nd, max_context_len)
            self.joined.record(self.side)
            cur.wait_event(self.joined)
        self.launches_per_step += 1

    def attend(self, num_seqs: int, max_context_len: int, chunks=None, new=None) -> None:
        """Attention over inputs already in self.q / self.tables / self.ctx
        (the device-resident path), output in self.out; current stream.
        chunks = (num_decode, num_chunks, max_chunk_len) runs rows past
        num_decode as prefill chunks (self.c_tables / c_ctx / c_start).
        new = (k_new, v_new, slot_mapping), one token per row at its newest
        position, is appended to the cache in the same launch."""
        S = num_seqs
        if chunks is not None:
            self._attend_mixed(self.slots_[0], S, max_context_len, chunks)
            return
        self._attend(self.q[:S], self.out[:S], self.tables[:S], self.ctx[:S], S, max_context_len, new)

    def step(self, q_host, k_new_host, v_new_host, slots_host, tables_host, ctx_host, out_host,
             max_context_len: int, chunks_host=None) -> torch.cuda.Event:
        """One decode step from pinned host buffers into pinned `out_host`.

        q_host [S, H, D]; k/v_new_host [T, Hkv, D]; slots_host int32 [T];
        tables_host int32 [S, max_blocks_per_seq]; ctx_host int32 [S].
        Asynchronous: returns the event after which `out_host` holds the
        result.  The host inputs may be rewritten once the next-but-one step
        has been submitted (or after synchronize()).
        chunks_host = (num_decode, query_start int32 [C+1], context_lens int32
        [C], block_tables int32 [C, max_blocks]): rows past num_decode are the
        query tokens of C prefill chunks (tables_host / ctx_host then describe
        the decode rows only).
        With fused_append and T == S, slot s must be the slot of row s's newest
        position (context_lens[s] - 1); a row whose slot is not is recorded as
        CF_DEVERR_SLOT and appends nothing.
        """
        S, T = q_host.shape[0], k_new_host.shape[0]
        b = self.slots_[self.n % len(self.slots_)]
        self.n += 1
        if b.used:
            self.h2d.wait_event(b.compute_done)  # the slot's inputs were read
        with torch.cuda.stream(self.h2d):
            b.q[:S].copy_(q_host, non_blocking=True)
            b.k_new[:T].copy_(k_new_host, non_blocking=True)
            b.v_new[:T].copy_(v_new_host, non_blocking=True)
            b.slots[:T].copy_(slots_host, non_blocking=True)
            nt = tables_host.shape[0]
            b.tables[:nt, : tables_host.shape[1]].copy_(tables_host, non_blocking=True)
            b.ctx[:nt].copy_(ctx_host, non_blocking=True)
            if chunks_host is not None:
                nd, qs, cc, ct = chunks_host
                nc = cc.shape[0]
                b.c_start[: nc + 1].copy_(qs, non_blocking=True)
                b.c_ctx[:nc].copy_(cc, non_blocking=True)
                b.c_tables[:nc, : ct.shape[1]].copy_(ct, non_blocking=True)
            b.h2d_done.record(self.h2d)
        self.stream.wait_event(b.h2d_done)
        if b.used:
            self.stream.wait_event(b.d2h_done)  # the slot's output was copied out
        fused = (self.fused_append or self.fp8) and chunks_host is None and T == S
        with torch.cuda.stream(self.stream):
            if not fused:
                if self.fp8:
                    ops.reshape_and_cache_fp8(b.k_new[:T], b.v_new[:T], self.k, self.v, b.slots[:T],
                                              *self.kv_scales)
                else:
                    ops.reshape_and_cache(b.k_new[:T], b.v_new[:T], self.k, self.v, b.slots[:T])
            if chunks_host is not None:
                nd, qs, cc, _ = chunks_host
                max_q = int((qs[1:] - qs[:-1]).max()) if cc.shape[0] else 0
                self._attend_mixed(b, S, max_context_len, (nd, cc.shape[0], max_q))
            else:
                self._attend(b.q[:S], b.out[:S], b.tables[:S], b.ctx[:S], S, max_context_len,
                             (b.k_new[:T], b.v_new[:T], b.slots[:T]) if fused else None)
            b.compute_done.record(self.stream)
        self.d2h.wait_event(b.compute_done)
        with torch.cuda.stream(self.d2h):
            out_host.copy_(b.out[:S], non_blocking=True)
            b.d2h_done.record(self.d2h)
        b.used = True
        return b.d2h_done

    def join(self) -> None:
        """Makes the compute stream wait for every submitted step's copies."""
        for b in self.slots_:
            if b.used:
                self.stream.wait_event(b.d2h_done)

    def synchronize(self) -> None:
        for s in (self.h2d, self.stream, self.d2h):
            s.synchronize()
