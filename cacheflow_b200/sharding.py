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

import copy
import heapq
import time
from contextlib import nullcontext
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


def _pairs(src, dst, device):
    import torch

    m = np.stack([np.asarray(src, np.int64), np.asarray(dst, np.int64)], 1)
    return torch.from_numpy(m).to(device)


def gather_blocks_cuda(cache, ids, out) -> None:
    """out[i] = cache[ids[i]] with the library's block-copy kernel."""
    from . import ops

    if len(ids) == 0:
        return
    ops.swap_blocks(cache, out, _pairs(ids, np.arange(len(ids)), cache.device), stream_tensor=cache)


def scatter_blocks_cuda(buf, cache, ids) -> None:
    """cache[ids[i]] = buf[i] with the library's block-copy kernel."""
    from . import ops

    if len(ids) == 0:
        return
    ops.swap_blocks(buf, cache, _pairs(np.arange(len(ids)), ids, cache.device), stream_tensor=cache)


def _clone(pool: LocalPool) -> LocalPool:
    """A copy whose later allocations and removals leave `pool` unchanged
    (the per-sequence id lists are replaced, never edited, so they are
    shared)."""
    q = copy.copy(pool)
    q.free = list(pool.free)
    q.tables = dict(pool.tables)
    q.lens = dict(pool.lens)
    return q


class MigrationError(RuntimeError):
    """A migration's transfers failed on this rank (the peer went away, or the
    deadline passed).  The transport has been aborted (with NCCL: the
    communicator, so every later collective on it fails at once instead of
    hanging), and this rank's pool bookkeeping is unchanged."""


class MigrationTimeout(MigrationError):
    """The transfers of a migration did not finish before its deadline."""


# migrate() calls made by this process: every rank makes the same calls, so
# the count names one call consistently across ranks.
_migrate_calls = 0


class P2PTransport:
    """Point-to-point transfers through torch.distributed: NCCL send/recv over
    NVLink between GPUs, gloo between CPU processes, posted as
    batch_isend_irecv groups."""

    def __init__(self, group=None, store=None):
        self.group = group
        self.store = store

    def check_peers(self, call: int, peers, timeout_s: float) -> None:
        """Host-side liveness check before anything is posted: this rank
        publishes a key for migration call `call` in the process group's
        store and waits, at most `timeout_s`, for the keys of the peers it
        exchanges with.  A peer that exited or never reaches the call raises
        MigrationError while no transfer of the call is on the device."""
        import datetime

        import torch.distributed as dist

        store = self.store if self.store is not None else dist.distributed_c10d._get_default_store()
        me = dist.get_rank()
        store.set(f"cf_migrate/{call}/{me}", "1")
        keys = [f"cf_migrate/{call}/{p}" for p in peers]
        try:
            store.wait(keys, datetime.timedelta(seconds=max(timeout_s, 1e-3)))
        except Exception as e:  # the store reports the timeout as a RuntimeError (or a subclass)
            missing = [p for p, k in zip(peers, keys) if not store.check([k])]
            raise MigrationError(f"migration call {call}: ranks {missing} did not arrive within "
                                 f"{timeout_s:g} s ({e})") from None

    def start(self, sends, recvs) -> list:
        """sends / recvs: lists of (tensor, peer rank).  Returns handles."""
        import torch.distributed as dist

        ops = [dist.P2POp(dist.isend, t, peer, self.group) for t, peer in sends]
        ops += [dist.P2POp(dist.irecv, t, peer, self.group) for t, peer in recvs]
        return dist.batch_isend_irecv(ops) if ops else []

    def wait(self, handles, timeout_s: float, poll_s: float = 2e-4) -> None:
        """Waits for every handle until the deadline; on expiry aborts and
        raises MigrationTimeout.  The host never blocks without a bound inside
        the communication library, so a peer that died or never sends cannot
        hang it.  NCCL handles are polled (is_completed() follows the device);
        gloo handles report completion only from wait(), which takes the
        remaining time as its own limit."""
        import datetime

        import torch.distributed as dist

        deadline = time.monotonic() + timeout_s
        if dist.get_backend(self.group) == "gloo":
            for i, h in enumerate(handles):
                left = deadline - time.monotonic()
                try:
                    if left <= 0:
                        raise RuntimeError("deadline passed")
                    h.wait(datetime.timedelta(seconds=left))
                except RuntimeError as e:
                    self.abort()
                    if time.monotonic() < deadline - 1e-3 and "deadline" not in str(e) and "imed out" not in str(e):
                        raise MigrationError(f"transfer {i} of {len(handles)} failed: {e}") from e
                    raise MigrationTimeout(f"{len(handles) - i} of {len(handles)} transfers unfinished after "
                                           f"{timeout_s:g} s") from None
            return
        pending = list(handles)
        while pending:
            try:
                pending = [h for h in pending if not h.is_completed()]
            except RuntimeError as e:  # the communicator reported an error
                self.abort()
                raise MigrationError(f"transfer failed: {e}") from e
            if not pending:
                break
            if time.monotonic() > deadline:
                self.abort()
                raise MigrationTimeout(f"{len(pending)} of {len(handles)} transfers unfinished after {timeout_s:g} s")
            time.sleep(poll_s)
        for h in handles:
            h.wait()  # orders the current CUDA stream after the transfer

    def abort(self) -> None:
        import torch.distributed as dist

        try:
            dist.distributed_c10d._abort_process_group(self.group or dist.group.WORLD)
        except Exception:  # gloo has no abort; the caller tears the group down
            pass


def migrate(moves, rank: int, pools: list[LocalPool], k_cache, v_cache,
            gather: Callable = gather_blocks_cuda, scatter: Callable = scatter_blocks_cuda,
            transport=None, timeout_s: float = 60.0, chunk_bytes: int = 1 << 30) -> dict:
    """Executes rebalance moves (seq, src rank, dst rank) with point-to-point
    transfers.  Every rank calls this with the same `moves`; `pools` is every
    rank's bookkeeping, kept identical on all ranks.

    The blocks a rank sends to one peer (its moved sequences' blocks, in move
    order) travel in chunks of at most `chunk_bytes` of K plus V (1 GiB: on
    two B200s 6 GB moved in 10.4 ms against 11.2 ms in 2 GiB chunks and
    15.3 ms as one group, where a chunk's gather, transfer and scatter run
    one after another): a sender
    gathers chunk i into a staging buffer (one block-copy launch per cache)
    and posts it in transfer group i, which holds chunk i of every pair this
    rank sends to or receives from; both ranks of a pair derive the same
    chunks from the shared bookkeeping, so chunk i of a pair is in group i on
    both sides and the groups complete in order without waiting on each
    other.  The gathers are all queued at once (NCCL orders each group after
    its gather), so later chunks' copies overlap earlier chunks' transfers;
    a receiver scatters chunk i into blocks allocated from its own pool as
    soon as group i has completed, on a side stream, while later groups are
    still in flight.  The host waits for each group with a deadline
    (`timeout_s` for the whole call): on expiry the transport is aborted and
    MigrationTimeout is raised with this rank's bookkeeping unchanged
    (MigrationError, its base, when a transfer fails before the deadline,
    e.g. because the peer exited); scatters already queued have then only
    written blocks that stay free.  Before any of that, the transport's
    check_peers (if it has one) confirms on the host, through the process
    group's store, that every peer of this rank reached the same call: a peer
    that exited between steps raises MigrationError with nothing posted.  On success every rank applies the moves
    to `pools`.  Returns {"blocks_sent", "blocks_received", "bytes_sent",
    "bytes_received", "device_ms", "host_ms", "groups"} for this rank (K and
    V; device_ms: CUDA events on the current stream from the first gather to
    the last scatter, None for CPU caches; host_ms: the whole call, the
    staging buffers' allocation included).

    gather / scatter move blocks between a cache and a contiguous staging
    buffer; the defaults are the library's CUDA kernels.
    """
    import torch

    t_host = time.perf_counter()
    deadline = time.monotonic() + timeout_s
    transport = transport or P2PTransport()
    # the new bookkeeping, applied to copies of the pools the moves touch:
    # destination ids are allocated in move order, identically on every rank
    touched = {r for _, a, b in moves for r in (a, b)}
    new = [(_clone(p) if r in touched else p) for r, p in enumerate(pools)]
    src_ids, dst_ids = {}, {}
    for seq, src, dst in moves:
        src_ids[seq] = list(new[src].tables[seq])
        dst_ids[seq] = new[dst].add_sequence(seq, new[src].lens[seq])
        new[src].remove_sequence(seq)

    tail = tuple(k_cache.shape[1:])
    block_bytes = k_cache[0].numel() * k_cache.element_size()
    cb = max(1, chunk_bytes // (2 * block_bytes))  # blocks per chunk (K and V)
    out_peers = sorted({d for _, s, d in moves if s == rank and d != rank})
    in_peers = sorted({s for _, s, d in moves if d == rank and s != rank})
    # per pair: the block ids in move order (sender: source ids; receiver:
    # destination ids) -- the same count on both sides
    out_ids = {p: np.fromiter((b for q, s, d in moves if s == rank and d == p for b in src_ids[q]), np.int64)
               for p in out_peers}
    in_ids = {p: np.fromiter((b for q, s, d in moves if s == p and d == rank for b in dst_ids[q]), np.int64)
              for p in in_peers}
    # every peer of this call alive (on the host) before anything is posted
    global _migrate_calls
    _migrate_calls += 1
    peers = sorted(set(out_peers) | set(in_peers))
    if peers and hasattr(transport, "check_peers"):
        transport.check_peers(_migrate_calls, peers, max(0.0, deadline - time.monotonic()))
    # staging buffers first: their allocation is host work, outside device_ms
    stage_out = {p: (torch.empty((len(i),) + tail, dtype=k_cache.dtype, device=k_cache.device),
                     torch.empty((len(i),) + tail, dtype=k_cache.dtype, device=k_cache.device))
                 for p, i in out_ids.items()}
    stage_in = {p: (torch.empty((len(i),) + tail, dtype=k_cache.dtype, device=k_cache.device),
                    torch.empty((len(i),) + tail, dtype=k_cache.dtype, device=k_cache.device))
                for p, i in in_ids.items()}
    nchunks = [-(-len(i) // cb) for i in list(out_ids.values()) + list(in_ids.values())]
    groups = max(nchunks, default=0)
    timed = k_cache.is_cuda
    side = None
    if timed:
        ev = [torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)]
        ev[0].record()
        if in_peers:
            side = torch.cuda.Stream(k_cache.device)
            side.wait_stream(torch.cuda.current_stream(k_cache.device))
    posted = []
    for g in range(groups):
        lo, hi = g * cb, (g + 1) * cb
        sends, recvs = [], []
        for p in out_peers:
            ids = out_ids[p][lo:hi]
            if len(ids):
                kb, vb = stage_out[p]
                gather(k_cache, ids, kb[lo:lo + len(ids)])
                gather(v_cache, ids, vb[lo:lo + len(ids)])
                sends += [(kb[lo:lo + len(ids)], p), (vb[lo:lo + len(ids)], p)]
        for p in in_peers:
            n = len(in_ids[p][lo:hi])
            if n:
                kr, vr = stage_in[p]
                recvs += [(kr[lo:lo + n], p), (vr[lo:lo + n], p)]
        try:
            posted.append(transport.start(sends, recvs))
        except RuntimeError as e:  # e.g. the peer aborted or exited already
            transport.abort()
            raise MigrationError(f"posting the transfers failed: {e}") from e
    for g, handles in enumerate(posted):
        transport.wait(handles, max(0.0, deadline - time.monotonic()))
        lo, hi = g * cb, (g + 1) * cb
        with torch.cuda.stream(side) if side is not None else nullcontext():
            for p in in_peers:
                ids = in_ids[p][lo:hi]
                if len(ids):
                    kr, vr = stage_in[p]
                    scatter(kr[lo:lo + len(ids)], k_cache, ids)
                    scatter(vr[lo:lo + len(ids)], v_cache, ids)
    if side is not None:
        torch.cuda.current_stream(k_cache.device).wait_stream(side)
    # local moves (src == dst) need no transfer: copy block by block
    for seq, src, dst in moves:
        if src == dst == rank:
            for cache in (k_cache, v_cache):
                tmp = torch.empty((len(src_ids[seq]),) + tail, dtype=cache.dtype, device=cache.device)
                gather(cache, src_ids[seq], tmp)
                scatter(tmp, cache, dst_ids[seq])
    device_ms = None
    if timed:
        ev[1].record()
        ev[1].synchronize()
        device_ms = ev[0].elapsed_time(ev[1])
    for p, q in zip(pools, new):
        if p is not q:
            p.__dict__.update(q.__dict__)
    n_out = sum(len(i) for i in out_ids.values())
    n_in = sum(len(i) for i in in_ids.values())
    return {"blocks_sent": n_out, "blocks_received": n_in, "bytes_sent": 2 * n_out * block_bytes,
            "bytes_received": 2 * n_in * block_bytes, "device_ms": device_ms, "groups": groups,
            "host_ms": (time.perf_counter() - t_host) * 1e3}
