"""Host logic of the multi-GPU sequence sharding: LPT assignment, per-rank
pools, rebalance planning, and block migration between two gloo ranks on CPU
(the CUDA block-copy kernels are swapped for CPU gathers here only)."""

import os
import socket

import numpy as np
import pytest

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
    out.copy_(cache[ids])


def _cpu_scatter(buf, cache, ids):
    cache[ids] = buf


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
    before = {s: (k[pools[rank].tables[s]].clone(), v[pools[rank].tables[s]].clone()) for s in pools[rank].tables}
    loads = [p.load() for p in pools]
    src = int(np.argmax(loads))
    dst = 1 - src
    seq = max(pools[src].tables, key=lambda s: pools[src].lens[s])
    moves = [(seq, src, dst)]
    sent = None
    if rank == src:
        sent = (k[pools[src].tables[seq]].clone(), v[pools[src].tables[seq]].clone())
    sharding.migrate(moves, rank, pools, k, v, gather=_cpu_gather, scatter=_cpu_scatter)
    if rank == src:
        torch.save(sent, os.path.join(result_dir, "sent.pt"))
    dist.barrier()
    if rank == dst:
        sk, sv = torch.load(os.path.join(result_dir, "sent.pt"))
        ids = pools[dst].tables[seq]
        ok = torch.equal(k[ids], sk) and torch.equal(v[ids], sv)
        # untouched sequences keep their blocks
        for s, (bk, bv) in before.items():
            ok = ok and torch.equal(k[pools[dst].tables[s]], bk) and torch.equal(v[pools[dst].tables[s]], bv)
        with open(os.path.join(result_dir, "ok"), "w") as f:
            f.write("1" if ok else "0")
    assert seq not in pools[src].tables and seq in pools[dst].tables
    dist.barrier()
    dist.destroy_process_group()


def test_block_migration_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp

    port = _free_port()
    mp.start_processes(_migration_worker, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn")
    assert (tmp_path / "ok").read_text() == "1"
