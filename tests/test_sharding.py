"""Host logic of the multi-GPU sequence sharding: LPT assignment, per-rank
pools, rebalance planning, and block migration between two gloo ranks on CPU
(the CUDA block-copy kernels are swapped for CPU gathers here only)."""

import copy
import os
import socket
import time

import numpy as np
import pytest
import torch

from cacheflow_b200 import sharding


def test_lpt_assignment_balances_kv_bytes():
    rng = np.random.default_rng(0)
    ctx = rng.integers(512, 32769, 1024)
    for world in (1, 2, 4, 8):
        parts = sharding.lpt_assign(ctx, world)
        assert sorted(np.concatenate(parts).tolist()) == list(range(1024))
        loads = [int(ctx[p].sum()) for p in parts]
        assert max(loads) - min(loads) <= ctx.max()
        assert max(loads) / (ctx.sum() / world) < 1.01


def test_pools_hold_disjoint_local_ids():
    rng = np.random.default_rng(1)
    ctx = rng.integers(16, 5000, 64)
    pools = sharding.shard_workload(ctx, 4, rng=rng)
    assert sum(len(p.tables) for p in pools) == 64
    for p in pools:
        ids = [b for t in p.tables.values() for b in t]
        assert len(ids) == len(set(ids)) and max(ids) < p.num_blocks
        seqs = sorted(p.tables)
        c, t = p.block_table(seqs)
        assert np.all((c + 15) // 16 <= t.shape[1])


def test_pool_exhaustion_raises():
    p = sharding.LocalPool(4)
    p.add_sequence(0, 48)
    with pytest.raises(MemoryError):
        p.add_sequence(1, 40)
    p.remove_sequence(0)
    p.add_sequence(1, 64)


def test_rebalance_plan_reduces_imbalance():
    loads = [1000, 100, 100, 100]
    lens = [{0: 400, 1: 300, 2: 200, 3: 100}, {4: 100}, {5: 100}, {6: 100}]
    moves = sharding.plan_rebalance(loads, lens, tolerance=0.1)
    after = list(loads)
    for s, a, b in moves:
        c = next(d[s] for d in lens if s in d)
        after[a] -= c
        after[b] += c
    assert max(after) - min(after) < max(loads) - min(loads)
    assert max(after) <= 500


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cpu_gather(cache, ids, out):
    out.copy_(cache[torch.as_tensor(np.asarray(ids, np.int64))])


def _cpu_scatter(buf, cache, ids):
    cache[torch.as_tensor(np.asarray(ids, np.int64))] = buf


def _migration_worker(rank, world, port, result_dir):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ctx = np.array([300, 50, 700, 20, 400, 90], np.int64)
    rng = np.random.default_rng(5)
    pools = sharding.shard_workload(ctx, world, pool_factor=3.0, rng=rng)  # room to receive
    shape = (max(p.num_blocks for p in pools) + 64, 2, 16, 8)
    g = torch.Generator().manual_seed(100 + rank)
    k = torch.randn(shape, generator=g)
    v = torch.randn(shape, generator=g)
    loads = [p.load() for p in pools]
    src = int(np.argmax(loads))
    dst = 1 - src
    # both directions in one call: the largest sequence of the loaded rank
    # one way, the smallest of the other rank back
    seq = max(pools[src].tables, key=lambda s: pools[src].lens[s])
    back = min(pools[dst].tables, key=lambda s: pools[dst].lens[s])
    moves = [(seq, src, dst), (back, dst, src)]
    stay = [s for s in pools[rank].tables if s not in (seq, back)]
    before = {s: (k[pools[rank].tables[s]].clone(), v[pools[rank].tables[s]].clone()) for s in stay}
    mine = seq if rank == src else back
    torch.save((k[pools[rank].tables[mine]].clone(), v[pools[rank].tables[mine]].clone()),
               os.path.join(result_dir, f"sent{rank}.pt"))
    stats = sharding.migrate(moves, rank, pools, k, v, gather=_cpu_gather, scatter=_cpu_scatter, timeout_s=60)
    dist.barrier()
    got = back if rank == src else seq
    sk, sv = torch.load(os.path.join(result_dir, f"sent{1 - rank}.pt"))
    ids = pools[rank].tables[got]
    ok = torch.equal(k[ids], sk) and torch.equal(v[ids], sv)
    # untouched sequences keep their blocks
    for s, (bk, bv) in before.items():
        ok = ok and torch.equal(k[pools[rank].tables[s]], bk) and torch.equal(v[pools[rank].tables[s]], bv)
    ok = ok and stats["blocks_received"] == len(ids) and stats["bytes_received"] == 2 * len(ids) * k[0].numel() * 4
    ok = ok and seq in pools[dst].tables and seq not in pools[src].tables
    ok = ok and back in pools[src].tables and back not in pools[dst].tables
    with open(os.path.join(result_dir, f"ok{rank}"), "w") as f:
        f.write("1" if ok else "0")
    dist.barrier()
    dist.destroy_process_group()


def test_block_migration_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp

    port = _free_port()
    mp.start_processes(_migration_worker, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn")
    assert (tmp_path / "ok0").read_text() == "1"
    assert (tmp_path / "ok1").read_text() == "1"


def _four_rank_plan(world):
    """The rebalancing round the bench runs at N > 1, on CPU: LPT shares,
    rank r loses 0.4 * r / (N - 1) of its sequences, then plan_rebalance."""
    ctx = np.random.default_rng(21).integers(20, 900, 48).astype(np.int64)
    pools = sharding.shard_workload(ctx, world, pool_factor=3.0, rng=np.random.default_rng(5))
    rng = np.random.default_rng(99)
    for r, p in enumerate(pools):
        seqs = sorted(p.tables)
        for s in rng.choice(seqs, int(0.4 * r / (world - 1) * len(seqs)), replace=False):
            p.remove_sequence(int(s))
    moves = sharding.plan_rebalance([p.load() for p in pools], [p.lens for p in pools], tolerance=0.02)
    return pools, moves


def _many_peer_worker(rank, world, port, result_dir, chunk_bytes):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    pools, moves = _four_rank_plan(world)
    shape = (max(p.num_blocks for p in pools) + 64, 2, 16, 8)
    g = torch.Generator().manual_seed(200 + rank)
    k, v = torch.randn(shape, generator=g), torch.randn(shape, generator=g)
    for s, a, b in moves:
        if a == rank:
            ids = pools[rank].tables[s]
            torch.save((k[ids].clone(), v[ids].clone()), os.path.join(result_dir, f"seq{s}.pt"))
    moved = {s for s, _, _ in moves}
    stay = [s for s in pools[rank].tables if s not in moved]
    before = {s: (k[pools[rank].tables[s]].clone(), v[pools[rank].tables[s]].clone()) for s in stay}
    stats = sharding.migrate(moves, rank, pools, k, v, gather=_cpu_gather, scatter=_cpu_scatter, timeout_s=60,
                             chunk_bytes=chunk_bytes)
    dist.barrier()
    ok = True
    got = 0
    for s, a, b in moves:
        if b == rank:
            sk, sv = torch.load(os.path.join(result_dir, f"seq{s}.pt"))
            ids = pools[rank].tables[s]
            ok = ok and torch.equal(k[ids], sk) and torch.equal(v[ids], sv)
            got += len(ids)
        ok = ok and (s in pools[b].tables) and (s not in pools[a].tables)
    for s, (bk, bv) in before.items():
        ok = ok and torch.equal(k[pools[rank].tables[s]], bk) and torch.equal(v[pools[rank].tables[s]], bv)
    ok = ok and stats["blocks_received"] == got
    with open(os.path.join(result_dir, f"ok{rank}"), "w") as f:
        f.write("1" if ok else "0")
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("chunk_bytes", [1 << 30, 3 * 1024])
def test_block_migration_four_gloo_ranks_many_peers(tmp_path, chunk_bytes):
    """plan_rebalance's moves between four ranks (several senders and
    receivers, some ranks both) through one migrate() call per rank: in one
    transfer group, and in chunks of one block (K and V: 2 KB of 3 KB), so
    every pair spans many groups of different counts."""
    import torch.multiprocessing as mp

    _, moves = _four_rank_plan(4)
    pairs = {(a, b) for _, a, b in moves}
    assert len(moves) >= 3 and len(pairs) >= 2, moves
    port = _free_port()
    mp.start_processes(_many_peer_worker, args=(4, port, str(tmp_path), chunk_bytes), nprocs=4,
                       start_method="spawn")
    for r in range(4):
        assert (tmp_path / f"ok{r}").read_text() == "1", r


class _RecordingTransport(sharding.P2PTransport):
    """Counts the transfer groups it is asked to post."""

    def __init__(self):
        super().__init__()
        self.posted = 0

    def start(self, sends, recvs):
        self.posted += 1
        return super().start(sends, recvs)


def _peer_gone_worker(rank, world, port, result_dir):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    dist.barrier()
    if rank == 1:
        os._exit(0)  # leaves between steps: nothing of it is in flight
    ctx = np.array([300, 50, 700, 20, 400, 90], np.int64)
    pools = sharding.shard_workload(ctx, world, pool_factor=3.0, rng=np.random.default_rng(5))
    shape = (max(p.num_blocks for p in pools) + 64, 2, 16, 8)
    k, v = torch.randn(shape), torch.randn(shape)
    seq = max(pools[0].tables, key=lambda s: pools[0].lens[s])
    before = {r: (dict(p.tables), dict(p.lens)) for r, p in enumerate(pools)}
    tr = _RecordingTransport()
    t0 = time.monotonic()
    try:
        sharding.migrate([(seq, 0, 1)], 0, pools, k, v, gather=_cpu_gather, scatter=_cpu_scatter, transport=tr,
                         timeout_s=2.0)
        res = "completed"
    except sharding.MigrationTimeout:
        res = "timeout"
    except sharding.MigrationError as e:
        res = "error" if "did not arrive" in str(e) else f"other error: {e}"
    unchanged = all(before[r] == (dict(p.tables), dict(p.lens)) for r, p in enumerate(pools))
    with open(os.path.join(result_dir, "r0"), "w") as f:
        f.write(f"{res} {tr.posted} {unchanged} {time.monotonic() - t0:.2f}")
    os._exit(0)  # no teardown with a peer that is gone


def test_migration_to_a_rank_that_left_fails_before_posting(tmp_path):
    """A peer that exited between steps: migrate() finds it missing in the
    process group's store, raises MigrationError within its deadline, posts
    no transfer and leaves the pools as they were."""
    import torch.multiprocessing as mp

    port = _free_port()
    mp.start_processes(_peer_gone_worker, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn")
    res, posted, unchanged, secs = (tmp_path / "r0").read_text().split()
    assert res == "error" and posted == "0" and unchanged == "True", (res, posted, unchanged)
    assert float(secs) < 10.0


class _DropSecondSend(sharding.P2PTransport):
    """Posts only the first of its sends: the V slice is lost on the way."""

    def start(self, sends, recvs):
        return super().start(sends[:1], recvs)


class _DelaySends(sharding.P2PTransport):
    """Posts its sends only after `delay` seconds."""

    def __init__(self, delay):
        super().__init__()
        self.delay = delay

    def start(self, sends, recvs):
        if sends:
            time.sleep(self.delay)
        return super().start(sends, recvs)


def _faulty_migration_worker(rank, world, port, result_dir, mode, delay, timeout_s):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ctx = np.array([300, 50, 700, 20, 400, 90], np.int64)
    pools = sharding.shard_workload(ctx, world, pool_factor=3.0, rng=np.random.default_rng(5))
    shape = (max(p.num_blocks for p in pools) + 64, 2, 16, 8)
    k = torch.randn(shape, generator=torch.Generator().manual_seed(100 + rank))
    v = torch.randn_like(k)
    src = int(np.argmax([p.load() for p in pools]))
    dst = 1 - src
    seq = max(pools[src].tables, key=lambda s: pools[src].lens[s])
    snapshot = copy.deepcopy(pools)
    transport = sharding.P2PTransport()
    if rank == src:
        transport = _DropSecondSend() if mode == "drop" else _DelaySends(delay)
    t0 = time.monotonic()
    try:
        sharding.migrate([(seq, src, dst)], rank, pools, k, v, gather=_cpu_gather, scatter=_cpu_scatter,
                         transport=transport, timeout_s=timeout_s if rank == dst else 60.0)
        outcome = "ok"
    except sharding.MigrationTimeout:
        outcome = "timeout"
    except sharding.MigrationError:
        outcome = "error"
    elapsed = time.monotonic() - t0
    unchanged = all(a.tables == b.tables and a.free == b.free for a, b in zip(pools, snapshot))
    with open(os.path.join(result_dir, f"r{rank}"), "w") as f:
        f.write(f"{outcome} {elapsed:.3f} {int(unchanged)} {int(rank == dst)}")
    # each rank stays up until the other has its result, so no transfer meets
    # a peer that has exited; both then leave without a group teardown (the
    # receiver's abandoned receive is still posted)
    flag = os.path.join(result_dir, f"r{1 - rank}")
    t1 = time.monotonic()
    while not os.path.exists(flag) and time.monotonic() - t1 < 60:
        time.sleep(0.05)
    os._exit(0)


def _run_faulty(tmp_path, mode, delay, timeout_s):
    import torch.multiprocessing as mp

    mp.start_processes(_faulty_migration_worker, args=(2, _free_port(), str(tmp_path), mode, delay, timeout_s),
                       nprocs=2, start_method="spawn")
    res = {}
    for r in (0, 1):
        outcome, elapsed, unchanged, is_dst = (tmp_path / f"r{r}").read_text().split()
        res["dst" if is_dst == "1" else "src"] = (outcome, float(elapsed), unchanged == "1")
    return res


def test_migration_dropped_transfer_times_out(tmp_path):
    """The sender loses its V slice: the receiver's wait ends at the deadline
    with MigrationTimeout and leaves its bookkeeping untouched."""
    res = _run_faulty(tmp_path, "drop", 0.0, 1.5)
    outcome, elapsed, unchanged = res["dst"]
    assert outcome == "timeout"
    assert 1.5 <= elapsed < 15
    assert unchanged


def test_migration_late_transfer_times_out(tmp_path):
    """The sender posts 6 s late, past the receiver's 1.5 s deadline: the
    receiver raises at its deadline, not when the data finally comes."""
    res = _run_faulty(tmp_path, "delay", 6.0, 1.5)
    outcome, elapsed, unchanged = res["dst"]
    assert outcome == "timeout"
    assert 1.5 <= elapsed < 5.5
    assert unchanged


def test_migration_late_transfer_within_deadline_completes(tmp_path):
    res = _run_faulty(tmp_path, "delay", 0.5, 20.0)
    assert res["dst"][0] == "ok" and not res["dst"][2]
    assert res["src"][0] == "ok"
