"""Sequence-sharded KV pools across GPUs, and block migration for rebalancing.

Each GPU (one process per GPU) owns one block pool and the sequences assigned
to it; block tables hold that pool's local ids, so decode attention needs no
communication at all.  Sequences are dealt by longest-processing-time on their
context length, which balances the KV bytes each GPU streams per step.

When the load drifts (sequences grow and finish at different rates), whole
sequences migrate: the sender gathers the sequence's K and V blocks into a
contiguous staging buffer with the library's block-copy kernel, ships it with
NCCL send/recv over NVLink, and the receiver scatters it into blocks it
allocates from its own pool and rewrites the sequence's table.  The transfer
lands in the receiver's own HBM first; nothing reads a peer's memory.

The host-side bookkeeping mirrors CacheFlow's BlockManager (free list of
physical ids, per-sequence block lists; src/cacheflow/kv_cache/
block_manager.cpp:35-79), partitioned per GPU.
"""

from __future__ import annotations

import heapq
from dataclasses import dataclass, field
from typing import Callable

import numpy as np

BLOCK = 16


def lpt_assign(context_lens: np.ndarray, world: int) -> list[np.ndarray]:
    """Sequence ids per rank: longest first onto the least-loaded rank."""
    order = np.argsort(-np.asarray(context_lens, np.int64), kind="stable")
    heap = [(0, r) for r in range(world)]
    out: list[list[int]] = [[] for _ in range(world)]
    for s in order:
        load, r = heapq.heappop(heap)
        out[r].append(int(s))
        heapq.heappush(heap, (load + int(context_lens[s]), r))
    return [np.array(sorted(x), np.int64) for x in out]


@dataclass
class LocalPool:
    """One GPU's block pool: free list of physical ids and per-sequence tables."""

    num_blocks: int
    free: list[int] = field(default_factory=list)
    tables: dict[int, list[int]] = field(default_factory=dict)  # seq id -> physical ids
    lens: dict[int, int] = field(default_factory=dict)  # seq id -> context length

    def __post_init__(self):
        if not self.free:
            self.free = list(range(self.num_blocks - 1, -1, -1))

    def allocate(self, n: int) -> list[int]:
        if n > len(self.free):
            raise MemoryError(f"pool exhausted: need {n} blocks, {len(self.free)} free")
        return [self.free.pop() for _ in range(n)]

    def add_sequence(self, seq: int, ctx: int) -> list[int]:
        ids = self.allocate((ctx + BLOCK - 1) // BLOCK)
        self.tables[seq] = ids
        self.lens[seq] = ctx
        return ids

    def remove_sequence(self, seq: int) -> list[int]:
        ids = self.tables.pop(seq)
        self.lens.pop(seq)
        self.free.extend(reversed(ids))
        return ids

    def load(self) -> int:
        return sum(self.lens.values())

    def block_table(self, seqs: list[int]) -> tuple[np.ndarray, np.ndarray]:
        """(context_lens int32 [S], block_tables int32 [S, max_blocks]) for `seqs`."""
        ctx = np.array([self.lens[s] for s in seqs], np.int32)
        mb = max(1, max((len(self.tables[s]) for s in seqs), default=1))
        t = np.zeros((len(seqs), mb), np.int32)
        for i, s in enumerate(seqs):
            t[i, : len(self.tables[s])] = self.tables[s]
        return ctx, t


def shard_workload(context_lens: np.ndarray, world: int, pool_factor: float = 1.2,
                   rng: np.random.Generator | None = None) -> list[LocalPool]:
    """Per-rank pools holding an LPT share of the sequences (ids shuffled)."""
    parts = lpt_assign(context_lens, world)
    pools = []
    for r in range(world):
        need = int(sum((int(context_lens[s]) + BLOCK - 1) // BLOCK for s in parts[r]))
        nb = max(1, int(np.ceil(pool_factor * need)))
        free = list(range(nb))
        if rng is not None:
            rng.shuffle(free)
        pool = LocalPool(nb, free=free)
        for s in parts[r]:
            pool.add_sequence(int(s), int(context_lens[s]))
        pools.append(pool)
    return pools


def plan_rebalance(loads: list[int], seq_lens: list[dict[int, int]], tolerance: float = 0.05):
    """Moves (seq, src rank, dst rank) that bring every rank within `tolerance`
    of the mean load, taking from the most loaded rank the largest sequence
    that does not overshoot."""
    loads = list(loads)
    lens = [dict(d) for d in seq_lens]
    mean = sum(loads) / max(1, len(loads))
    moves = []
    for _ in range(sum(len(d) for d in lens)):
        hi = max(range(len(loads)), key=lambda r: loads[r])
        lo = min(range(len(loads)), key=lambda r: loads[r])
        gap = loads[hi] - loads[lo]
        if loads[hi] <= mean * (1 + tolerance) or gap <= 0:
            break
        cand = [(c, s) for s, c in lens[hi].items() if c < gap]
        if not cand:
            break
        c, s = max(cand)
        moves.append((s, hi, lo))
        lens[hi].pop(s)
        lens[lo][s] = c
        loads[hi] -= c
        loads[lo] += c
    return moves


def gather_blocks_cuda(cache, ids: list[int], out) -> None:
    """out[i] = cache[ids[i]] with the library's block-copy kernel."""
    import torch

    from . import ops

    m = torch.tensor([[b, i] for i, b in enumerate(ids)], dtype=torch.int64, device=cache.device)
    ops.swap_blocks(cache, out, m, stream_tensor=cache)


def scatter_blocks_cuda(buf, cache, ids: list[int]) -> None:
    """cache[ids[i]] = buf[i] with the library's block-copy kernel."""
    import torch

    from . import ops

    m = torch.tensor([[i, b] for i, b in enumerate(ids)], dtype=torch.int64, device=cache.device)
    ops.swap_blocks(buf, cache, m, stream_tensor=cache)


def migrate(moves, rank: int, pools: list[LocalPool], k_cache, v_cache,
            gather: Callable = gather_blocks_cuda, scatter: Callable = scatter_blocks_cuda) -> None:
    """Executes rebalance moves with point-to-point sends (every rank calls this
    with the same `moves`; `pools` is every rank's bookkeeping, kept in sync).

    gather / scatter move blocks between the cache and a contiguous staging
    buffer; the defaults are the library's CUDA kernels.
    """
    import torch
    import torch.distributed as dist

    for seq, src, dst in moves:
        # Bookkeeping is deterministic, so every rank applies it identically.
        src_ids = list(pools[src].tables[seq])
        dst_ids = pools[dst].add_sequence(seq, pools[src].lens[seq])
        pools[src].remove_sequence(seq)
        shape = (len(src_ids),) + tuple(k_cache.shape[1:])
        if rank == src:
            kb = torch.empty(shape, dtype=k_cache.dtype, device=k_cache.device)
            vb = torch.empty_like(kb)
            gather(k_cache, src_ids, kb)
            gather(v_cache, src_ids, vb)
            if k_cache.is_cuda:
                torch.cuda.current_stream(k_cache.device).synchronize()
            reqs = [dist.P2POp(dist.isend, kb, dst), dist.P2POp(dist.isend, vb, dst)]
            for w in dist.batch_isend_irecv(reqs):
                w.wait()
        elif rank == dst:
            kb = torch.empty(shape, dtype=k_cache.dtype, device=k_cache.device)
            vb = torch.empty_like(kb)
            reqs = [dist.P2POp(dist.irecv, kb, src), dist.P2POp(dist.irecv, vb, src)]
            for w in dist.batch_isend_irecv(reqs):
                w.wait()
            scatter(kb, k_cache, dst_ids)
            scatter(vb, v_cache, dst_ids)
