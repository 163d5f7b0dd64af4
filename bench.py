"""Benchmark of the paged KV-cache decode path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload llama2_7b_ragged_decode] [--v1-split on|off]

A step is one decode step of the workload over resident HBM inputs:
reshape_and_cache of the new tokens, then paged attention (v1 for contexts
<= 8192 tokens, else v2 + reduce), plus copy_blocks for workloads with COW
forks.  The metric is KV bytes read per step (each (token, KV head) K and V
row once) / step time, in GB/s, summed over ranks; tokens/s (decode rows per
second per layer) is reported beside it.

Multi-GPU (torchrun, one process per GPU): every rank owns its own block pool
and no collective touches the data path.  Most workloads scale weakly (every
rank runs the workload's shape on its own seeded batch); llama3_70b_sharded
scales strongly (one 1024-sequence batch dealt to the ranks' pools by
longest-processing-time) and also times its pool operations (4 GB of swap to
and from pinned host memory, compaction of a half-freed pool).  Timing is CUDA
events on the launching stream, max over ranks.

--impl reference runs CacheFlow's own CPU decode step (oracle/_ref, built
from the reference sources) on a bounded sample of the same workload on the
host cores; under torchrun only rank 0 runs it.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from cacheflow_b200 import workloads  # noqa: E402

METRIC = "Paged decode attn: HBM GB/s (% of peak), tokens/s at 1/2/4/8 B200"
UNIT = "GB/s"
DTYPE_NAME = {"f32": "f32", "f16": "f16", "bf16": "bf16"}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def hbm_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ---------------------------------------------------------------------------
# Clock sampling during the timed region (nvidia-smi, 50 ms period).
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,utilization.gpu,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", str(self.idx)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, mx, reasons, loaded = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 10:
                continue
            try:
                clk, cmax, util = float(f[1]), float(f[2]), float(f[3])
            except ValueError:
                continue
            mx = cmax
            sm.append(clk)
            if util > 0:
                loaded.append(clk)
            for n, v in zip(names, f[6:10]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        use = loaded or sm
        return {"sm_mhz": statistics.median(use) if use else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm), "samples_under_load": len(loaded)}


# ---------------------------------------------------------------------------
# Our arm.
# ---------------------------------------------------------------------------
def fill_normal_(t, std, gen):
    return t.normal_(0.0, std, generator=gen)


def fill_fp8_(t, std, scale, gen, chunk=1 << 28):
    """float8_e4m3fn cache of N(0, std) values stored as e4m3(x / scale)."""
    import torch

    flat = t.view(-1)
    for i in range(0, flat.numel(), chunk):
        n = min(chunk, flat.numel() - i)
        x = torch.empty(n, dtype=torch.float32, device=t.device).normal_(0.0, std, generator=gen)
        flat[i:i + n] = (x / scale).to(torch.float8_e4m3fn)
    return t


SHARDED = {"llama3_70b_sharded"}
L2_BYTES = 126 * 1024 * 1024
L2_FLUSH_BYTES = 512 * 1024 * 1024


def rank_workload(args, rank: int, world: int):
    """This rank's batch and the scaling mode.

    Sharded workloads (strong scaling): one global batch, sequences dealt to
    ranks by longest-processing-time on context length, each rank's share
    re-homed into its own pool.  The others (weak scaling): every rank runs
    the workload's full shape on its own seeded batch.
    """
    from cacheflow_b200 import sharding

    kw = {"num_seqs": args.num_seqs} if args.num_seqs else {}
    if args.workload in SHARDED:
        full = workloads.make(args.workload, seed=1234, **kw)
        rows = sharding.lpt_assign(full.context_lens, world)[rank]
        return full.rehome(rows, seed=1234 + rank), "strong"
    # same batch shape on every rank (equal work per GPU); the cache contents
    # are seeded per rank
    return workloads.make(args.workload, seed=1234, **kw), "weak"


def time_pool_ops(w, k_cache, v_cache, world: int, swap_gb: float):
    """Timings of the block-movement operators on this rank's pool (the 70B
    configuration's per-step swap and compaction), CUDA events on the current
    stream:
      swap_out / swap_in  swap_gb / world GB of K blocks to / from pinned host
                          memory with the SM copy kernel (cf_swap_blocks);
      swap_out_dma        the same through the copy engines (cf_swap_blocks_dma);
      block_ops_swap_out / block_ops_swap_in
                          the same bytes as K and V pairs through
                          cf_execute_block_ops (host pair lists);
      compact             compaction of the pool after half of its sequences
                          are freed (cf_compaction_plan + cf_compact_kv_cache).
    """
    import torch

    from cacheflow_b200 import ops

    dev = k_cache.device
    res = {}
    block_bytes = k_cache[0].numel() * k_cache.element_size()
    nblk = (w.context_lens.astype(np.int64) + 15) // 16
    live = np.concatenate([w.block_tables[s, : nblk[s]] for s in range(w.num_seqs)])
    n = int(min(len(live), (swap_gb / world) * (1 << 30) // block_bytes))
    rng = np.random.default_rng(7)
    ids = rng.choice(live, n, replace=False).astype(np.int64)
    host = torch.empty((n,) + tuple(k_cache.shape[1:]), dtype=k_cache.dtype, pin_memory=True)
    out_map = torch.from_numpy(np.stack([ids, np.arange(n)], 1)).to(dev)
    in_map = torch.from_numpy(np.stack([np.arange(n), ids], 1)).to(dev)
    host_map = np.stack([ids, np.arange(n)], 1)

    def timed(fn, reps=3):
        fn()
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize(dev)
        return a.elapsed_time(b) / reps

    nbytes = n * block_bytes
    ms = timed(lambda: ops.swap_blocks(k_cache, host, out_map, stream_tensor=k_cache))
    res["swap_out"] = {"bytes": nbytes, "ms": round(ms, 3), "GB/s": round(nbytes / ms / 1e6, 1)}
    ms = timed(lambda: ops.swap_blocks(host, k_cache, in_map, stream_tensor=k_cache))
    res["swap_in"] = {"bytes": nbytes, "ms": round(ms, 3), "GB/s": round(nbytes / ms / 1e6, 1)}
    ms = timed(lambda: ops.swap_blocks_dma(k_cache, host, host_map, stream_tensor=k_cache), reps=1)
    res["swap_out_dma"] = {"bytes": nbytes, "ms": round(ms, 3), "GB/s": round(nbytes / ms / 1e6, 1),
                           "note": "random block ids: one copy per block"}
    # the scheduler's form of the same traffic: n/2 scattered (GPU, CPU) pairs
    # of K and V blocks through cf_execute_block_ops (host pair lists)
    h = n // 2
    hk, hv = host[:h], host[h:2 * h]
    so = np.ascontiguousarray(np.stack([ids[:h], np.arange(h)], 1))
    si = np.ascontiguousarray(np.stack([np.arange(h), ids[:h]], 1))
    ms = timed(lambda: ops.execute_block_ops(k_cache, v_cache, hk, hv, swaps_out=so))
    res["block_ops_swap_out"] = {"bytes": 2 * h * block_bytes, "ms": round(ms, 3),
                                 "GB/s": round(2 * h * block_bytes / ms / 1e6, 1),
                                 "note": "cf_execute_block_ops, K and V, random block ids"}
    ms = timed(lambda: ops.execute_block_ops(k_cache, v_cache, hk, hv, swaps_in=si))
    res["block_ops_swap_in"] = {"bytes": 2 * h * block_bytes, "ms": round(ms, 3),
                                "GB/s": round(2 * h * block_bytes / ms / 1e6, 1),
                                "note": "cf_execute_block_ops, K and V, random block ids"}
    del host, hk, hv
    keep = rng.random(w.num_seqs) < 0.5
    used = np.zeros(w.num_blocks, np.uint8)
    for s in np.flatnonzero(keep):
        used[w.block_tables[s, : nblk[s]]] = 1
    src, dst = ops.compaction_plan(used)
    s_t, d_t = torch.from_numpy(src).to(dev), torch.from_numpy(dst).to(dev)
    moved = 2 * len(src) * 2 * block_bytes  # read + write, K and V
    ms = timed(lambda: ops.compact_kv_cache(k_cache, v_cache, s_t, d_t), reps=1)
    res["compact"] = {"moves": int(len(src)), "bytes_read_written": moved, "ms": round(ms, 3),
                      "GB/s": round(moved / ms / 1e6, 1)}
    return res


def workload_config(args, w, world: int, scaling: str, seqs_total: int) -> dict:
    """The `config` of the bench line: the workload this rank's share runs
    (both arms print the same dict; implementation choices of this library
    go to `impl_config`)."""
    fp8 = args.kv_dtype == "fp8"
    kv_step = (w.kv_bytes() // w.elem_bytes if fp8 else
               (w.chunked_kv_bytes() if w.has_chunks and args.prefill == "chunked" else w.kv_bytes()))
    flush = w.kv_bytes() < 4 * L2_BYTES
    return {
        "workload": w.name,
        "num_seqs_per_gpu": w.num_seqs,
        "num_seqs_total": int(seqs_total),
        "num_heads": w.num_heads,
        "num_kv_heads": w.num_kv_heads,
        "head_dim": w.head_dim,
        "block_size": 16,
        "context_lens": "min %d / mean %.0f / max %d" % (w.context_lens.min(), w.context_lens.mean(),
                                                          w.context_lens.max()),
        "pool_blocks_per_gpu": w.num_blocks,
        "kv_dtype": "fp8 e4m3" if fp8 else w.dtype,
        "kv_bytes_per_step_per_gpu": kv_step,
        "unique_kv_bytes_per_step_per_gpu": w.unique_kv_bytes() // (w.elem_bytes if fp8 else 1),
        "l2": ("L2 flushed before every timed step (512 MB write, then a 512 MB read of a clean buffer; outside "
               "the step's events)" if flush and args.l2_clean == "on" else
               "L2 flushed before every timed step (512 MB write, outside the step's events)" if flush else
               "inputs larger than L2 (%.2f GB of KV read per step per GPU vs 126 MB L2)" % (kv_step / 1e9)),
        "parallelism": (f"dp{world} (one global batch, sequences dealt to per-GPU pools by LPT)"
                        if scaling == "strong" else
                        f"dp{world} (per-GPU pools and batches, no data-path collective)"),
    }


def measure(args, w, rank: int, world: int, dev, kernel: str, steps: int, warmup: int, e2e: bool = True,
            post=None) -> dict:
    """Times `steps` decode steps of workload `w` on this rank (after `warmup`
    untimed ones) and, with e2e, the same step through DecodeEngine.step from
    pinned host buffers.  Every timed attention launch is bracketed by CUDA
    events on the engine's stream.  post(k_cache, v_cache) runs after the
    timings with the caches still resident and its result is returned as
    "post".  Collectives: barriers only (the caller all-reduces)."""
    import torch
    import torch.distributed as dist

    from cacheflow_b200 import ops
    from cacheflow_b200.engine import DecodeEngine

    local = dev.index
    tdt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[w.dtype]
    gen = torch.Generator(device=dev)
    gen.manual_seed(4321 + rank)
    S, H, Hkv, D = w.num_seqs, w.num_heads, w.num_kv_heads, w.head_dim
    fp8 = args.kv_dtype == "fp8"
    if fp8 and (w.dtype == "f32" or w.has_chunks):
        raise SystemExit("--kv-dtype fp8 needs a 16-bit decode-only workload")
    kv_scale = w.std / 64.0  # N(0, std) / scale: 7 sigma reaches the e4m3 maximum (448)
    if fp8:
        k_cache = torch.empty(w.cache_shape(), dtype=torch.float8_e4m3fn, device=dev)
        v_cache = torch.empty_like(k_cache)
        fill_fp8_(k_cache, w.std, kv_scale, gen)
        fill_fp8_(v_cache, w.std, kv_scale, gen)
    else:
        k_cache = torch.empty(w.cache_shape(), dtype=tdt, device=dev)
        v_cache = torch.empty_like(k_cache)
        fill_normal_(k_cache, w.std, gen)
        fill_normal_(v_cache, w.std, gen)
    T = len(w.slot_mapping)
    q = torch.empty((S, H, D), dtype=tdt, device=dev).normal_(0, w.std, generator=gen)
    k_new = torch.empty((T, Hkv, D), dtype=tdt, device=dev).normal_(0, w.std, generator=gen)
    v_new = torch.empty_like(k_new).normal_(0, w.std, generator=gen)
    slots = torch.from_numpy(w.slot_mapping).to(dev)
    tables = torch.from_numpy(w.block_tables).to(dev)
    ctx = torch.from_numpy(w.context_lens).to(dev)
    pairs = torch.from_numpy(w.copy_pairs).to(dev) if len(w.copy_pairs) else None
    mctx = w.max_context_len

    chunked = w.has_chunks and args.prefill == "chunked"
    nc = len(w.chunk_context_lens) if chunked else 0
    # decode-only batches (one new token per row, at its newest position)
    # append it inside the attention launch unless --append separate
    fused = (args.append == "fused" or (args.append == "auto" and not fp8)) and not w.has_chunks and T == S
    new_rows = (k_new, v_new, slots) if fused else None
    engine = DecodeEngine(k_cache, v_cache, H, S, w.block_tables.shape[1], T, split_v1=(args.v1_split == "on"),
                          kernel=kernel, max_chunks=nc, fused_append=fused,
                          kv_scales=(kv_scale, kv_scale) if fp8 else None, query_dtype=tdt)
    engine.q[:S].copy_(q)
    engine.tables.copy_(tables)
    engine.ctx.copy_(ctx)
    stream = engine.stream
    chunks = None
    kv_step = w.kv_bytes() // w.elem_bytes if fp8 else w.kv_bytes()  # fp8: one byte per element
    if chunked:
        # decode rows [0, num_decode) through paged attention, the prefill
        # chunks' tokens through the multi-query operator
        nd = w.num_decode
        engine.c_tables[:, : w.chunk_block_tables.shape[1]].copy_(torch.from_numpy(w.chunk_block_tables))
        engine.c_ctx.copy_(torch.from_numpy(w.chunk_context_lens))
        engine.c_start.copy_(torch.from_numpy(w.chunk_query_start))
        max_q = int(np.diff(w.chunk_query_start).max())
        chunks = (nd, nc, max_q)
        mctx = int(w.context_lens[:nd].max())
        kv_step = w.chunked_kv_bytes()

    att_ev = []
    # batches that fit in L2 (126 MB) are timed with L2 overwritten between steps
    flush = (torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
             if w.kv_bytes() < 4 * L2_BYTES else None)
    # After the write, a read of a second (clean) buffer leaves L2 holding
    # clean lines only, so the timed step does not also pay for writing the
    # flush buffer's dirty lines back to HBM (--l2-clean off keeps them).
    flush_clean = (torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
                   if flush is not None and args.l2_clean == "on" else None)

    def step(record=False):
        if pairs is not None:
            ops.copy_blocks(k_cache, v_cache, pairs)
        if fused:
            pass
        elif fp8:
            ops.reshape_and_cache_fp8(k_new, v_new, k_cache, v_cache, slots, kv_scale, kv_scale)
        else:
            ops.reshape_and_cache(k_new, v_new, k_cache, v_cache, slots)
        if record:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            engine.attend(S, mctx, chunks, new_rows)
            b.record(stream)
            att_ev.append((a, b))
        else:
            engine.attend(S, mctx, chunks, new_rows)

    with torch.cuda.stream(stream):
        for _ in range(warmup):
            step()
        launches_per_step = engine.launches_per_step + (0 if fused else 1) + (1 if pairs is not None else 0)
        torch.cuda.synchronize(dev)
        if ops.device_errors(local) != 0:
            raise RuntimeError("device error word set during warm-up")
        if world > 1:
            dist.barrier()
        clocks = ClockSampler(local) if rank == 0 else None
        if clocks:
            clocks.start()
            time.sleep(0.25)
        # the GPU idled while the sampler started: bring its clocks back up
        # with a few more untimed steps before the timed region
        for _ in range(3):
            step()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        step_ev = []
        t0.record(stream)
        for i in range(steps):
            if flush is not None:
                # the batch fits in L2: overwrite L2 before every step and time
                # the steps alone
                flush.zero_()
                if flush_clean is not None:
                    flush_clean.max()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                step(record=True)
                b.record(stream)
                step_ev.append((a, b))
            else:
                # every timed attention launch is bracketed by its own events
                step(record=True)
        t1.record(stream)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        clock_info = clocks.stop() if clocks else None
    if flush is not None:
        ms_step = sum(a.elapsed_time(b) for a, b in step_ev) / len(step_ev)
    else:
        ms_step = t0.elapsed_time(t1) / steps
    att_ms = sum(a.elapsed_time(b) for a, b in att_ev) / len(att_ev)
    if ops.device_errors(local) != 0:
        raise RuntimeError("device error word set during the timed region")

    e2e_ms = None
    if e2e:
        # e2e through the public engine API with pinned host buffers.
        nrows = chunks[0] if chunked else S  # rows described by block tables / context lengths
        pin = dict(
            q=q.cpu().pin_memory(), k=k_new.cpu().pin_memory(), v=v_new.cpu().pin_memory(),
            s=slots.cpu().pin_memory(), t=tables[:nrows].cpu().pin_memory(), c=ctx[:nrows].cpu().pin_memory(),
            o=torch.empty((S, H, D), dtype=tdt).pin_memory())
        chunks_host = None
        if chunked:
            chunks_host = (chunks[0], torch.from_numpy(w.chunk_query_start).pin_memory(),
                           torch.from_numpy(w.chunk_context_lens).pin_memory(),
                           torch.from_numpy(w.chunk_block_tables).pin_memory())
        for _ in range(max(3, warmup // 4)):
            engine.step(pin["q"], pin["k"], pin["v"], pin["s"], pin["t"], pin["c"], pin["o"], mctx, chunks_host)
        engine.synchronize()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        engine.h2d.wait_event(e0)  # the copy streams start inside the timed region too
        engine.d2h.wait_event(e0)
        e2e_steps = max(1, steps // 2)
        for _ in range(e2e_steps):
            engine.step(pin["q"], pin["k"], pin["v"], pin["s"], pin["t"], pin["c"], pin["o"], mctx, chunks_host)
        engine.join()  # the last output copy ends the region
        e1.record(stream)
        torch.cuda.synchronize(dev)
        e2e_ms = e0.elapsed_time(e1) / e2e_steps
        if ops.device_errors(local) != 0:
            raise RuntimeError("device error word set during the end-to-end region")

    alg_bytes = kv_step + w.qo_bytes() + w.table_bytes()
    if fused:  # the appended rows: new K/V read, cache rows written, slots read
        alg_bytes += 2 * T * Hkv * D * (k_new.element_size() + k_cache.element_size()) + 4 * T
    res = {
        "ms_step": ms_step, "att_ms": att_ms, "e2e_ms": e2e_ms, "kv_step": kv_step, "alg_bytes": alg_bytes,
        "launches_per_step": launches_per_step, "clocks": clock_info, "fused": fused, "fp8": fp8,
        "kv_scale": kv_scale, "chunked": chunked, "chunks": chunks, "flush": flush is not None,
        "flush_clean": flush_clean is not None, "v2": engine._use_v2(mctx), "split": engine.workspace is not None,
        "attention_launches": len(att_ev),
        "h2d_bytes": engine.h2d_bytes(S, T), "d2h_bytes": engine.d2h_bytes(S),
    }
    if flush is not None:
        res["copy_same_traffic"] = cold_copy_time(stream, alg_bytes, flush, flush_clean)
    if post is not None:
        with torch.cuda.stream(stream):
            res["post"] = post(k_cache, v_cache)
    del engine, k_cache, v_cache, flush, flush_clean
    torch.cuda.empty_cache()
    return res


def cold_copy_time(stream, traffic: int, flush, flush_clean, reps: int = 50) -> dict:
    """A device copy moving the same DRAM traffic (half read, half written)
    as one attention launch, timed like the steps of a batch that fits in L2
    (L2 overwritten before each copy, events around the copy alone): what any
    kernel can reach at this size from a cold L2."""
    import torch

    n = traffic // 2 // 16 * 16
    src = torch.empty(n, dtype=torch.uint8, device=flush.device)
    dst = torch.empty_like(src)
    src.fill_(1)
    times = []
    with torch.cuda.stream(stream):
        for i in range(reps + 5):
            flush.zero_()
            if flush_clean is not None:
                flush_clean.max()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            dst.copy_(src)
            b.record(stream)
            times.append((a, b))
    torch.cuda.synchronize(flush.device)
    ms = sorted(a.elapsed_time(b) for a, b in times[5:])
    med = ms[len(ms) // 2]
    return {"bytes": 2 * n, "us": round(med * 1e3, 2), "GBps": round(2 * n / (med * 1e-3) / 1e9, 1)}


def attention_kind(r: dict) -> str:
    if r["v2"]:
        return "v2 (512-token partitions) + reduce"
    return "v1" + (" (split into partitions, merged by a reduce kernel)" if r["split"] else "")


def side_config(args, name: str, rank: int, world: int, dev, peak: float) -> dict:
    """One more workload timed at N=1 beside the headline, once with the
    library's v1 split and once with the reference's kernel choice."""
    w = workloads.make(name, seed=1234)
    out = {"workload": name, "num_seqs": w.num_seqs, "num_heads": w.num_heads, "num_kv_heads": w.num_kv_heads,
           "head_dim": w.head_dim, "dtype": w.dtype,
           "context_lens": "min %d / mean %.0f / max %d" % (w.context_lens.min(), w.context_lens.mean(),
                                                             w.context_lens.max())}
    for kernel in ("v1", "reference"):
        r = measure(args, w, rank, world, dev, kernel, args.steps, args.warmup, e2e=False)
        if r["att_ms"] > r["ms_step"] * 1.0001:
            raise RuntimeError(f"{name}: attention time {r['att_ms']} ms above the step time {r['ms_step']} ms")
        achieved = r["alg_bytes"] / (r["att_ms"] * 1e-3) / 1e9
        out["v1_split" if kernel == "v1" else "reference_kernel"] = {
            "attention": attention_kind(r),
            "value": round(r["kv_step"] / (r["ms_step"] * 1e-3) / 1e9, 1),
            "unit": UNIT,
            "ms_per_step": round(r["ms_step"], 4),
            "kernel_ms": round(r["att_ms"], 4),
            "achieved": round(achieved, 1),
            "frac": round(achieved / peak, 4),
            "alg_bytes_per_launch": r["alg_bytes"],
            "tokens_per_s": round(w.num_seqs / (r["ms_step"] * 1e-3), 1),
            "clocks": r["clocks"],
        }
    return out


def rebalance_check(full, parts, rank: int, world: int, k_cache, v_cache) -> dict:
    """A rebalancing round after the timed steps (strong-scaled workload, N>1):
    every rank rebuilds all ranks' pool bookkeeping from the same LPT shares,
    a seeded fraction of each rank's sequences finishes (rank r loses up to
    40 % of them, growing with r), plan_rebalance moves sequences from the
    loaded ranks to the light ones, and migrate() ships their blocks over
    NCCL.  Timed with CUDA events on this rank's stream (gather -> transfers
    -> scatter); the caller takes the max over ranks.  Then every moved
    sequence's attention is computed on its receiver and compared bitwise
    with what the sender computed before the move."""
    import torch
    import torch.distributed as dist

    from cacheflow_b200 import ops, sharding

    dev = k_cache.device
    pools = []
    for r in range(world):
        wr = full.rehome(parts[r], seed=1234 + r)
        nblk = (wr.context_lens.astype(np.int64) + 15) // 16
        tabs = {int(g): [int(b) for b in wr.block_tables[i, : nblk[i]]] for i, g in enumerate(parts[r])}
        used = {b for t in tabs.values() for b in t}
        free = [b for b in range(wr.num_blocks - 1, -1, -1) if b not in used]
        pools.append(sharding.LocalPool(wr.num_blocks, free=free, tables=tabs,
                                        lens={int(g): int(c) for g, c in zip(parts[r], wr.context_lens)}))
    rng = np.random.default_rng(99)
    for r, p in enumerate(pools):
        seqs = sorted(p.tables)
        frac = 0.4 * r / max(1, world - 1)
        for s in rng.choice(seqs, int(frac * len(seqs)), replace=False):
            p.remove_sequence(int(s))
    loads = [p.load() for p in pools]
    moves = sharding.plan_rebalance(loads, [p.lens for p in pools], tolerance=0.02)
    after = list(loads)
    for s, a, b in moves:
        c = pools[a].lens[s]
        after[a] -= c
        after[b] += c

    def attend(pool, seqs, qq):
        c, t = pool.block_table(seqs)
        tt, cc = torch.from_numpy(t).to(dev), torch.from_numpy(c).to(dev)
        mc = int(c.max())
        ws = None
        n = ops.paged_attention_v1_workspace_size(qq, k_cache, tt, mc)
        if n:
            ws = torch.empty((n,), dtype=torch.uint8, device=dev)
        o = torch.empty_like(qq)
        ops.paged_attention_v1(o, qq, k_cache, v_cache, tt, cc, None, mc, workspace=ws)
        return o

    H = full.num_heads
    qdt = k_cache.dtype
    out_seqs = {}
    for peer in range(world):
        seqs = [s for s, a, b in moves if a == rank and b == peer]
        if seqs:
            g = torch.Generator(device=dev).manual_seed(777 + rank)
            qq = torch.empty((len(seqs), H, full.head_dim), dtype=qdt, device=dev).normal_(0, full.std, generator=g)
            out_seqs[peer] = (seqs, qq, attend(pools[rank], seqs, qq))
    # NCCL connects a pair of ranks at its first point-to-point transfer (a
    # one-time cost per process): connect the pairs the moves use first
    pairs = sorted({(a, b) for _, a, b in moves if a != b})
    tr = sharding.P2PTransport()
    tr.wait(tr.start([(torch.zeros(1, device=dev), b) for a, b in pairs if a == rank],
                     [(torch.empty(1, device=dev), a) for a, b in pairs if b == rank]), 60.0)
    torch.cuda.synchronize(dev)
    dist.barrier()
    stats = sharding.migrate(moves, rank, pools, k_cache, v_cache, timeout_s=60.0)
    torch.cuda.synchronize(dev)
    ms = stats["device_ms"]
    # verification traffic (not timed): each sender ships the queries and the
    # outputs it computed; the receiver recomputes on its new blocks
    sends, recvs, checks = [], [], []
    for peer, (seqs, qq, oo) in out_seqs.items():
        sends += [(qq, peer), (oo, peer)]
    for peer in range(world):
        seqs = [s for s, a, b in moves if a == peer and b == rank]
        if seqs:
            qq = torch.empty((len(seqs), H, full.head_dim), dtype=qdt, device=dev)
            oo = torch.empty_like(qq)
            recvs += [(qq, peer), (oo, peer)]
            checks.append((seqs, qq, oo))
    tr.wait(tr.start(sends, recvs), 60.0)
    verified = mismatched = 0
    for seqs, qq, oo in checks:
        got = attend(pools[rank], seqs, qq)
        for i in range(len(seqs)):
            verified += 1
            mismatched += int(not torch.equal(got[i], oo[i]))
    torch.cuda.synchronize(dev)
    t = torch.tensor([ms, stats["bytes_sent"], verified, mismatched, ops.device_errors(dev.index)],
                     dtype=torch.float64, device=dev)
    tmax = torch.tensor([ms, stats["host_ms"]], dtype=torch.float64, device=dev)
    dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    (ms_max, host_max), sent = tmax.tolist(), t[1].item()
    verified, mismatched, errs = int(t[2].item()), int(t[3].item()), t[4].item()
    return {
        "moves": len(moves),
        "bytes": int(sent),
        "ms": round(ms_max, 3),
        "GB/s": round(sent / (ms_max * 1e-3) / 1e9, 1) if ms_max > 0 else None,
        "host_ms": round(host_max, 1),
        "load_before": [int(x) for x in loads],
        "load_after": [int(x) for x in after],
        "sequences_verified": verified,
        "bitwise_equal": mismatched == 0 and errs == 0,
        "how": ("seeded finishes (rank r loses 0.4*r/(N-1) of its sequences), plan_rebalance to 2 %, "
                "migrate(): block-copy gather, NCCL send/recv into the receiver's HBM, scatter, pipelined in 1 GiB "
                "chunks (rank pairs connected "
                "beforehand by a 1-element exchange); ms = CUDA events from the first gather to the last scatter "
                "on each rank, max over ranks (host_ms: the whole call, bookkeeping included); moved sequences' "
                "attention recomputed on the receiver"),
    }


def run_ours(args):
    import torch
    import torch.distributed as dist

    from cacheflow_b200 import _lib, sharding

    rank, world, local = dist_env()
    _lib.load()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    w, scaling = rank_workload(args, rank, world)
    fp8 = args.kv_dtype == "fp8"

    def post(k_cache, v_cache):
        extra = {}
        if args.workload in SHARDED and not args.no_pool_ops and not fp8:
            extra["pool_ops"] = time_pool_ops(w, k_cache, v_cache, world, args.swap_gb)
        if world > 1 and scaling == "strong" and not args.no_migration and not fp8:
            full = workloads.make(args.workload, seed=1234, **({"num_seqs": args.num_seqs} if args.num_seqs else {}))
            parts = sharding.lpt_assign(full.context_lens, world)
            extra["migration"] = rebalance_check(full, parts, rank, world, k_cache, v_cache)
        return extra

    r = measure(args, w, rank, world, dev, args.kernel, args.steps, args.warmup, e2e=True, post=post)
    ms_step, att_ms, e2e_ms = r["ms_step"], r["att_ms"], r["e2e_ms"]
    if att_ms > ms_step * 1.0001:
        raise RuntimeError(f"attention time {att_ms} ms above the step time {ms_step} ms")
    pool_ops = r["post"].get("pool_ops")
    if pool_ops is not None:
        keys = sorted(pool_ops)
        ms_t = torch.tensor([pool_ops[k]["ms"] for k in keys], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
        for k, m in zip(keys, ms_t.tolist()):
            b = pool_ops[k].get("bytes", pool_ops[k].get("bytes_read_written"))
            pool_ops[k]["all_ranks_GB/s"] = round(world * b / m / 1e6, 1)

    S, H, Hkv, D = w.num_seqs, w.num_heads, w.num_kv_heads, w.head_dim
    kv_step = r["kv_step"]
    times = torch.tensor([ms_step, att_ms, e2e_ms], dtype=torch.float64, device=dev)
    totals = torch.tensor([kv_step, S], dtype=torch.float64, device=dev)
    # per-rank spread: what limits the scaling (the slowest rank sets the step)
    spread = torch.tensor([att_ms, kv_step, -att_ms, -kv_step], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
        dist.all_reduce(totals, op=dist.ReduceOp.SUM)
        dist.all_reduce(spread, op=dist.ReduceOp.MAX)
    ms_step, att_ms, e2e_ms = times.tolist()
    kv_total, seqs_total = totals.tolist()
    k_max, b_max, k_min, b_min = spread[0].item(), spread[1].item(), -spread[2].item(), -spread[3].item()

    if rank == 0:
        peak, peak_kind = hbm_peak()
        alg_bytes = r["alg_bytes"]
        achieved = alg_bytes / (att_ms * 1e-3) / 1e9
        value = kv_total / (ms_step * 1e-3) / 1e9
        chunks = r["chunks"]
        line = {
            "metric": METRIC,
            "value": round(value, 1),
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_step, 4),
            "higher_is_better": True,
            "scaling": scaling,
            "vs_baseline": None,
            "dtype": DTYPE_NAME[w.dtype],
            "data": "synthetic (seeded N(0,%g) caches, shapes of the workload)" % w.std,
            "config": workload_config(args, w, world, scaling, seqs_total),
            "impl_config": {
                "prefill": ("chunked: %d decode rows + %d chunks through the multi-query operator"
                            % (chunks[0], chunks[1]) if r["chunked"] else
                            ("one decode row per prefill token" if w.has_chunks else None)),
                "attention": attention_kind(r),
                "kernel_choice": args.kernel,
                "v1_split": args.v1_split,
                "append": ("new K/V appended inside the attention launch" if r["fused"]
                           else "reshape_and_cache launch before attention"),
                "kv_cache": ("fp8 e4m3, per-cache scale %g (f16 tensor-core / f32 FMA arithmetic)" % r["kv_scale"]
                             if fp8 else w.dtype),
            },
            "tokens_per_s": round(seqs_total / (ms_step * 1e-3), 1),
            "unique_kv_GBps": round(world * w.unique_kv_bytes() / (w.elem_bytes if fp8 else 1)
                                    / (ms_step * 1e-3) / 1e9, 1),
            "frac_of_hbm_peak": round(value / (peak * world), 4),
            "roofline": {
                "bound": "hbm",
                "kernel": ("paged_attention" + ("_v2+reduce" if r["v2"] else "_v1")
                           + ("+paged_prefill" if r["chunked"] else "")),
                "achieved": round(achieved, 1),
                "peak": peak,
                "unit": "GB/s",
                "frac": round(achieved / peak, 4),
                "peak_source": peak_kind,
                "alg_bytes_per_launch": alg_bytes,
                "kernel_ms": round(att_ms, 4),
                "kernel_launches_timed": r["attention_launches"],
                # the committed captures are of 1-GPU launches: a strong-scaled
                # rank's launch is another shape
                "traffic": (traffic_from_profiles(w.name + ("_fp8" if fp8 else ""))
                            if world == 1 or scaling == "weak" else None),
            },
            "e2e": {
                "value": round(kv_total / (e2e_ms * 1e-3) / 1e9, 1),
                "unit": UNIT,
                "ms_per_step": round(e2e_ms, 4),
                "h2d_bytes_per_step": r["h2d_bytes"],
                "d2h_bytes_per_step": r["d2h_bytes"],
                "api": "cacheflow_b200.engine.DecodeEngine.step (pinned host in, pinned host out)",
            },
            "gpu_launches": r["launches_per_step"] * args.steps,
            "clocks": r["clocks"],
        }
        if world > 1:
            line["ranks"] = {
                "kernel_ms_min": round(k_min, 4),
                "kernel_ms_max": round(k_max, 4),
                "kv_bytes_max_over_mean": round(b_max / (kv_total / world), 6),
                "kv_bytes_min_over_mean": round(b_min / (kv_total / world), 6),
                "note": ("the step is the slowest rank's; spread of the attention launch time and of the KV "
                         "bytes each rank reads"),
            }
        if "copy_same_traffic" in r:
            c = r["copy_same_traffic"]
            line["roofline"]["cold_copy_same_traffic"] = {
                **c, "frac_of_peak": round(c["GBps"] / peak, 4), "kernel_over_copy": round(att_ms * 1e3 / c["us"], 3),
                "note": ("a device copy of the launch's algorithmic bytes (half read, half written) timed like the "
                         "step, L2 overwritten before each: the reachable rate at this size"),
            }
        if pool_ops is not None:
            line["pool_ops_rank0"] = pool_ops
        if "migration" in r["post"]:
            line["migration"] = r["post"]["migration"]
    if world == 1 and args.side_configs != "none" and not fp8:
        line["configs"] = {name: side_config(args, name, rank, world, dev, peak)
                           for name in args.side_configs.split(",") if name != args.workload}
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(w, budget_s=args.cpu_seconds)
            line["cpu_port"] = cpu_port_baseline(w)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def traffic_from_profiles(workload: str):
    """DRAM bytes per launch of the attention kernel from a committed ncu summary, if any."""
    p = ROOT / "profiles" / f"traffic_{workload}.json"
    if p.exists():
        try:
            return json.loads(p.read_text()).get("dram_bytes_per_launch")
        except Exception:
            return None
    return None


# ---------------------------------------------------------------------------
# CacheFlow's own CPU decode step on a bounded sample (reference arm / baseline).
# ---------------------------------------------------------------------------
def reference_sample(w: workloads.Workload, max_seqs: int, max_tokens: int | None = None):
    """The first `max_seqs` rows of the workload (each context cut to its
    first `max_tokens` tokens, if given) with their blocks renumbered into a
    compact fp32 pool (the reference is fp32-only)."""
    rows = np.arange(min(max_seqs, w.num_seqs))
    ctx = w.context_lens[rows].astype(np.int64)
    if max_tokens is not None:
        ctx = np.minimum(ctx, max_tokens)
    nblk = (ctx + 15) // 16
    tables = np.zeros((len(rows), int(nblk.max())), np.int32)
    remap = {}
    for i, r in enumerate(rows):
        for b in range(nblk[i]):
            old = int(w.block_tables[r, b])
            tables[i, b] = remap.setdefault(old, len(remap))
    return ctx.astype(w.context_lens.dtype), tables, len(remap)


def cpu_baseline(w: workloads.Workload, budget_s: float = 15.0, steps: int | None = None, warmup: int = 1,
                 max_seqs: int = 16, total_budget_s: float | None = None):
    """CacheFlow's own CPU decode step on the first rows of `w`.  With
    `steps`, exactly that many timed steps run; total_budget_s then caps the
    whole run (warm-up included) by cutting the sample's contexts shorter
    (the rows stay, so every host thread keeps a sequence: the reference
    step spreads sequences over its threads), found from one probe step;
    only contexts already at 16 tokens make it drop rows.  Without `steps`,
    steps repeat for about budget_s seconds."""
    from oracle import oracle

    threads = os.cpu_count() or 1
    n = min(w.num_seqs, max_seqs)
    cap = None
    while True:
        ctx, tables, pool = reference_sample(w, n, cap)
        ref = oracle.RefCpu(w.num_heads, w.num_kv_heads, w.head_dim, pool, threads)
        k, v = ref.caches()
        rng = np.random.default_rng(7)
        k[...] = rng.standard_normal(k.shape, dtype=np.float32) * np.float32(w.std)
        v[...] = rng.standard_normal(v.shape, dtype=np.float32) * np.float32(w.std)
        ref.set_batch(ctx, tables)
        if steps is None or total_budget_s is None:
            break
        t_probe = ref.step()
        if t_probe * (steps + warmup) <= total_budget_s or (n == 1 and int(ctx.max()) <= 16):
            break
        ref.close()
        f = total_budget_s / (t_probe * (steps + warmup))
        longest = int(ctx.max())
        if longest > 16:
            cap = max(16, min(longest - 16, int(longest * f * 0.9)))
        else:
            n = max(1, min(n - 1, int(n * f)))
    try:
        for _ in range(warmup):
            ref.step()
        times = []
        t_start = time.perf_counter()
        while True:
            times.append(ref.step())
            if steps is not None:
                if len(times) >= steps:
                    break
            elif time.perf_counter() - t_start > budget_s:
                break
    finally:
        ref.close()
    t = sum(times) / len(times)
    sample_bytes = int(ctx.astype(np.int64).sum()) * 2 * w.num_kv_heads * w.head_dim * w.elem_bytes
    cut = f", contexts cut to their first {cap} tokens" if cap is not None else ""
    return {
        "value": round(sample_bytes / t / 1e9, 3),
        "unit": UNIT,
        "cores": threads,
        "kind": "reference",
        "sample": (f"CacheFlow BatchDecodeEngine::step, CPU build (batch_decode.cpp:33-88,190-240; fp32, "
                   f"reads K only, no output) on the first {len(ctx)} of {w.num_seqs} sequences of {w.name}"
                   f"{cut} ({int(ctx.sum())} tokens), {len(times)} steps of {t*1e3:.1f} ms, {threads} threads; "
                   f"value = that sample's {w.dtype} KV bytes / step time"),
        "tokens_per_s": round(len(ctx) / t, 2),
    }


def cpu_port_baseline(w: workloads.Workload, max_seqs: int = 16, max_tokens: int = 2048,
                      budget_s: float = 4.0) -> dict:
    """The oracle's C restatement of the decode step (correct softmax
    attention in f64, one pass per query head over its KV head's blocks, the
    reference kernel's loop order) on the first `max_seqs` rows of `w`, each
    context cut to its first `max_tokens` tokens, timed with all host threads
    (repeated for about `budget_s`) and with one."""
    import math

    from oracle import oracle

    threads = os.cpu_count() or 1
    rng = np.random.default_rng(11)
    code = oracle.BF16 if w.dtype == "bf16" else None
    ctx, tables, pool = reference_sample(w, min(w.num_seqs, max_seqs), max_tokens)
    q = workloads.host_values((len(ctx), w.num_heads, w.head_dim), w.dtype, w.std, rng)
    k = workloads.host_values((pool, w.num_kv_heads, 16, w.head_dim), w.dtype, w.std, rng)
    v = workloads.host_values((pool, w.num_kv_heads, 16, w.head_dim), w.dtype, w.std, rng)
    scale = 1.0 / math.sqrt(w.head_dim)
    times = {}
    for nt in (threads, 1):
        t0 = time.perf_counter()
        reps = 0
        while True:
            oracle.paged_attention(q, k, v, tables, ctx, scale, code, num_threads=nt)
            reps += 1
            if nt == 1 or time.perf_counter() - t0 > budget_s or reps >= 50:
                break
        times[nt] = (time.perf_counter() - t0) / reps
    kv_bytes = int(ctx.astype(np.int64).sum()) * 2 * w.num_kv_heads * w.head_dim * w.elem_bytes
    return {
        "value": round(kv_bytes / times[threads] / 1e9, 3),
        "value_one_thread": round(kv_bytes / times[1] / 1e9, 3),
        "unit": UNIT,
        "cores": threads,
        "kind": "port",
        "sample": (f"the oracle's C restatement (oracle/cf_oracle.c cfo_paged_attention: f64 softmax attention, "
                   f"per query head over its KV head's blocks) on the first {len(ctx)} of {w.num_seqs} sequences "
                   f"of {w.name}, contexts cut to their first {max_tokens} tokens ({int(ctx.sum())} tokens): "
                   f"{times[threads]*1e3:.1f} ms per step on {threads} threads, {times[1]*1e3:.1f} ms on one; "
                   f"value = the sample's {w.dtype} KV bytes / step time"),
    }


def run_reference(args):
    rank, world, local = dist_env()
    if rank != 0:
        return
    # this rank's share of the workload, as the GPU arm's rank 0 runs it
    w, scaling = rank_workload(args, 0, world)
    seqs_total = workloads.make(args.workload, seed=1234,
                                **({"num_seqs": args.num_seqs} if args.num_seqs else {})).num_seqs \
        if scaling == "strong" else w.num_seqs * world
    cb = cpu_baseline(w, steps=args.steps, warmup=args.warmup, total_budget_s=args.cpu_total_seconds)
    line = {
        "metric": METRIC,
        "value": cb["value"],
        "unit": UNIT,
        "impl": "reference",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "higher_is_better": True,
        "scaling": scaling,
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,%g) caches, shapes of the workload)" % w.std,
        "config": workload_config(args, w, world, scaling, seqs_total),
        "tokens_per_s": cb["tokens_per_s"],
        "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="llama3_70b_sharded", choices=sorted(workloads.WORKLOADS))
    ap.add_argument("--side-configs", default="llama3_8b_long_decode",
                    help="comma-separated workloads also timed at N=1 (v1 split and the reference's kernel "
                         "choice), reported under 'configs'; 'none' to skip")
    ap.add_argument("--v1-split", choices=["on", "off"], default="on")
    ap.add_argument("--kernel", choices=["v1", "reference"], default="v1",
                    help="decode attention: v1 with the library's context split at every length, or the "
                         "reference's choice (v1 up to 8192 tokens, v2 with 512-token partitions beyond)")
    ap.add_argument("--num-seqs", type=int, default=0,
                    help="override the workload's sequence count (small profiling cases)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-pool-ops", action="store_true", help="skip swap / compaction timings")
    ap.add_argument("--no-migration", action="store_true",
                    help="N>1 strong scaling: skip the rebalancing round (NCCL block migration)")
    ap.add_argument("--l2-clean", choices=["on", "off"], default="on",
                    help="small batches: read a clean buffer after the L2-flush write")
    ap.add_argument("--kv-dtype", choices=["native", "fp8"], default="native",
                    help="KV cache element type: the workload's own, or fp8 e4m3 with a per-cache scale")
    ap.add_argument("--append", choices=["auto", "fused", "separate"], default="auto",
                    help="decode batches: append the new K/V inside the attention launch, or run "
                         "reshape_and_cache before it (auto: fused for 16-bit caches, separate for fp8, "
                         "the faster of the two on each)")
    ap.add_argument("--prefill", choices=["chunked", "rows"], default="chunked",
                    help="prefill tokens of mixed batches: multi-query chunks or one decode row each")
    ap.add_argument("--swap-gb", type=float, default=4.0, help="GB swapped out and in (whole job)")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--cpu-total-seconds", type=float, default=120.0,
                    help="--impl reference: cap on the whole run; the sample shrinks to fewer rows to fit")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
