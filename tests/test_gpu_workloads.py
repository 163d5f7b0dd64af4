"""Every benchmark workload at its full size on the GPU, checked through
properties that do not depend on size plus the oracle on a subset of rows:

* the new K/V rows land bit-exactly in their slots (reshape_and_cache);
* COW copies make destination blocks equal their sources (copy_blocks);
* attention of a subset of rows (longest, shortest, random) matches the CPU
  oracle run on just the blocks those rows read;
* v1, split v1 and v2 agree on the whole batch;
* the 70B-shaped pool: a swap-out / swap-in round trip through pinned host
  memory is bit-exact, and compaction of a pool with half its blocks freed
  moves every live block intact (per-block checksums) and leaves attention
  over the remapped tables bitwise unchanged.
"""

import math

import numpy as np
import pytest

from cacheflow_b200 import workloads
from helpers import CODE, TOL, as_f64, assert_close

pytestmark = pytest.mark.gpu

NAMES = ["cpu_decode_fp32", "llama2_7b_ragged_decode", "llama3_8b_long_decode", "continuous_batching_mixed",
         "llama3_70b_sharded"]


def _attention(ops, w, st, mode):
    import torch

    S, H, D = w.num_seqs, w.num_heads, w.head_dim
    out = torch.empty((S, H, D), dtype=st["q"].dtype, device=st["q"].device)
    mctx = w.max_context_len
    args = (st["q"], st["k_cache"], st["v_cache"], st["tables"], st["ctx"], 1.0 / math.sqrt(D), mctx)
    if mode == "v1":
        ops.paged_attention_v1(out, *args)
    elif mode == "v1split":
        n = ops.paged_attention_v1_workspace_size(st["q"], st["k_cache"], st["tables"], mctx)
        ws = torch.empty(max(n, 16), dtype=torch.uint8, device=out.device)
        ops.paged_attention_v1(out, *args, workspace=ws)
    else:
        P = ops.v2_num_partitions(mctx)
        es = torch.empty((S, H, P), device=out.device)
        ml = torch.empty_like(es)
        tmp = torch.empty((S, H, P, D), device=out.device)
        ops.paged_attention_v2(out, es, ml, tmp, *args)
    return out


def _free():
    import gc

    import torch

    gc.collect()
    torch.cuda.empty_cache()


@pytest.mark.parametrize("name", NAMES)
def test_full_size_workload(cflib, oracle_mod, name):
    import torch

    from cacheflow_b200 import ops

    w = workloads.make(name)
    st = workloads.device_state(w, "cuda")
    try:
        if st["pairs"] is not None:
            ops.copy_blocks(st["k_cache"], st["v_cache"], st["pairs"])
            src, dst = st["pairs"][:, 0], st["pairs"][:, 1]
            assert torch.equal(st["k_cache"][dst], st["k_cache"][src])
            assert torch.equal(st["v_cache"][dst], st["v_cache"][src])
        ops.reshape_and_cache(st["k_new"], st["v_new"], st["k_cache"], st["v_cache"], st["slots"])
        slots = st["slots"].long()
        assert torch.equal(st["k_cache"][slots // 16, :, slots % 16], st["k_new"])
        assert torch.equal(st["v_cache"][slots // 16, :, slots % 16], st["v_new"])

        main = "v1" if w.max_context_len <= 8192 else "v2"
        out = _attention(ops, w, st, main)
        rng = np.random.default_rng(0)
        rows = np.unique(np.concatenate([[np.argmax(w.context_lens), np.argmin(w.context_lens)],
                                         rng.choice(w.num_seqs, 2, replace=False)]))
        q, k, v, tables, ctx = workloads.gather_rows_for_oracle(w, st, rows)
        want = oracle_mod.paged_attention(q, k, v, tables, ctx, 1.0 / math.sqrt(w.head_dim), CODE[w.dtype],
                                          num_threads=8)
        assert_close(as_f64(out[torch.from_numpy(rows).cuda()]), want, w.dtype, f"{name} rows {rows.tolist()}")

        # all attention paths agree on the whole batch (each within TOL of the
        # truth, so within twice that of each other)
        atol, rtol = TOL[w.dtype]
        for mode in ("v1", "v1split", "v2"):
            if mode == main:
                continue
            other = _attention(ops, w, st, mode)
            err = (other.double() - out.double()).abs()
            lim = 2 * atol + 2 * rtol * out.double().abs()
            assert bool((err <= lim).all()), f"{name}: {mode} vs {main} max err {err.max().item():.3e}"
            del other
        if w.has_chunks:
            # the prefill chunks through the multi-query operator agree with
            # their per-token decode rows
            nd = w.num_decode
            pre = torch.empty_like(out[nd:])
            ops.paged_prefill_attention(pre, st["q"][nd:], st["k_cache"], st["v_cache"],
                                        torch.from_numpy(w.chunk_block_tables).cuda(),
                                        torch.from_numpy(w.chunk_context_lens).cuda(),
                                        torch.from_numpy(w.chunk_query_start).cuda())
            ref = out[nd:].double()
            err = (pre.double() - ref).abs()
            assert bool((err <= 2 * atol + 2 * rtol * ref.abs()).all()), f"chunked prefill max err {err.max().item():.3e}"
        assert ops.device_errors(0) == 0
    finally:
        del st
        _free()


def test_70b_pool_swap_round_trip_and_compaction(cflib):
    import torch

    from cacheflow_b200 import _lib, ops

    w = workloads.make("llama3_70b_sharded")
    st = workloads.device_state(w, "cuda")
    kc, vc = st["k_cache"], st["v_cache"]
    block_bytes = kc[0].numel() * kc.element_size()
    try:
        rng = np.random.default_rng(1)
        nblk = (w.context_lens.astype(np.int64) + 15) // 16
        live = np.concatenate([w.block_tables[s, : nblk[s]] for s in range(w.num_seqs)])

        # swap 4 GB of K blocks out to pinned host memory and back
        n_swap = min(len(live), (4 << 30) // block_bytes)
        ids = rng.choice(live, n_swap, replace=False)
        host = torch.empty((n_swap,) + tuple(kc.shape[1:]), dtype=kc.dtype, pin_memory=True)
        saved = kc[torch.from_numpy(ids).cuda()].clone()
        out_map = torch.from_numpy(np.stack([ids, np.arange(n_swap)], 1).astype(np.int64)).cuda()
        in_map = torch.from_numpy(np.stack([np.arange(n_swap), ids], 1).astype(np.int64)).cuda()
        ops.swap_blocks(kc, host, out_map, stream_tensor=kc)
        ops.memset_blocks(kc, torch.from_numpy(ids.astype(np.int32)).cuda())
        ops.swap_blocks(host, kc, in_map, stream_tensor=kc)
        torch.cuda.synchronize()
        assert torch.equal(kc[torch.from_numpy(ids).cuda()], saved)
        del saved, host
        _free()

        # free half of the sequences, compact the pool, check every live block moved intact
        keep = rng.random(w.num_seqs) < 0.5
        used = np.zeros(w.num_blocks, np.uint8)
        for s in np.flatnonzero(keep):
            used[w.block_tables[s, : nblk[s]]] = 1
        src, dst = ops.compaction_plan(used)
        assert ops.check_compaction_plan(src, dst, w.num_blocks) == _lib.CF_OK

        def checksums(t):
            # per-block sum of the 16-bit patterns, 16K blocks at a time (an
            # int32 sum of one block cannot overflow: 16,384 values < 2^15)
            n = t.shape[0]
            out = torch.empty(n, dtype=torch.int32, device=t.device)
            flat = t.view(torch.int16).view(n, -1)
            for i in range(0, n, 16384):
                out[i:i + 16384] = flat[i:i + 16384].to(torch.int32).sum(1, dtype=torch.int32)
            return out

        ck, cv = checksums(kc), checksums(vc)
        q_rows = np.flatnonzero(keep)
        sub = w.subset(q_rows)
        st_sub = dict(st)
        st_sub.update(q=st["q"][torch.from_numpy(q_rows).cuda()].contiguous(),
                      tables=torch.from_numpy(sub.block_tables).cuda(), ctx=torch.from_numpy(sub.context_lens).cuda())
        before = _attention(ops, sub, st_sub, "v2")

        ops.compact_kv_cache(kc, vc, torch.from_numpy(src).cuda(), torch.from_numpy(dst).cuda())
        ck2, cv2 = checksums(kc), checksums(vc)
        s_t, d_t = torch.from_numpy(src.astype(np.int64)).cuda(), torch.from_numpy(dst.astype(np.int64)).cuda()
        assert torch.equal(ck2[d_t], ck[s_t]) and torch.equal(cv2[d_t], cv[s_t])
        stay = torch.from_numpy(np.flatnonzero(used[: used.sum()]).astype(np.int64)).cuda()
        assert torch.equal(ck2[stay], ck[stay])

        remap = np.arange(w.num_blocks, dtype=np.int32)
        remap[src] = dst
        sub.block_tables = remap[sub.block_tables]
        st_sub["tables"] = torch.from_numpy(sub.block_tables).cuda()
        after = _attention(ops, sub, st_sub, "v2")
        assert torch.equal(after, before)
        assert ops.device_errors(0) == 0
    finally:
        del st, kc, vc
        _free()
