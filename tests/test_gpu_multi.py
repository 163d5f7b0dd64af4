"""Sequence migration between two GPUs: blocks gathered with the library's
block-copy kernel, shipped with NCCL send/recv into the receiver's own HBM,
scattered into newly allocated blocks; attention of the migrated sequence on
the receiver is bitwise identical to what the sender computed before."""

import os
import socket

import numpy as np
import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _attend_one(ops, pool, seq, k, v, q):
    import torch

    ctx, tab = pool.block_table([seq])
    out = torch.empty_like(q)
    ops.paged_attention_v1(out, q, k, v, torch.from_numpy(tab).to(k.device), torch.from_numpy(ctx).to(k.device),
                           None, int(ctx.max()))
    return out


def _worker(rank, world, port, result_dir):
    import datetime

    import torch
    import torch.distributed as dist

    from cacheflow_b200 import ops, sharding

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        ctx = np.array([3000, 700, 5000, 120, 2600, 900, 4100, 33], np.int64)
        pools = sharding.shard_workload(ctx, world, pool_factor=3.0, rng=np.random.default_rng(5))
        nb = max(p.num_blocks for p in pools)
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        k = torch.randn((nb, 8, 16, 128), generator=g, device=dev).to(torch.bfloat16)
        v = torch.randn((nb, 8, 16, 128), generator=g, device=dev).to(torch.bfloat16)
        q = torch.randn((1, 32, 128), generator=torch.Generator(device=dev).manual_seed(7), device=dev).to(torch.bfloat16)
        loads = [p.load() for p in pools]
        src = int(np.argmax(loads))
        dst = 1 - src
        seq = max(pools[src].tables, key=lambda s: pools[src].lens[s])
        if rank == src:
            before = _attend_one(ops, pools[src], seq, k, v, q)
            torch.save(before.cpu(), os.path.join(result_dir, "before.pt"))
        sharding.migrate([(seq, src, dst)], rank, pools, k, v)
        torch.cuda.synchronize(dev)
        dist.barrier()
        if rank == dst:
            after = _attend_one(ops, pools[dst], seq, k, v, q).cpu()
            before = torch.load(os.path.join(result_dir, "before.pt"))
            ok = torch.equal(after, before) and ops.device_errors(rank) == 0
            with open(os.path.join(result_dir, "ok"), "w") as f:
                f.write("1" if ok else "0")
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_sequence_migration_over_nccl(cflib, tmp_path):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    assert (tmp_path / "ok").read_text() == "1"


def _worker_both_ways(rank, world, port, result_dir):
    import datetime

    import torch
    import torch.distributed as dist

    from cacheflow_b200 import ops, sharding

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        rng = np.random.default_rng(11)
        ctx = rng.integers(30, 6000, 24)
        pools = sharding.shard_workload(ctx, world, pool_factor=3.0, rng=np.random.default_rng(12))
        nb = max(p.num_blocks for p in pools)
        g = torch.Generator(device=dev).manual_seed(200 + rank)
        k = torch.randn((nb, 8, 16, 128), generator=g, device=dev).to(torch.bfloat16)
        v = torch.randn((nb, 8, 16, 128), generator=g, device=dev).to(torch.bfloat16)
        # three sequences each way in one call
        out0 = sorted(pools[0].tables, key=lambda s: -pools[0].lens[s])[:3]
        out1 = sorted(pools[1].tables, key=lambda s: pools[1].lens[s])[:3]
        moves = [(s, 0, 1) for s in out0] + [(s, 1, 0) for s in out1]
        mine = out0 if rank == 0 else out1
        qg = torch.Generator(device=dev).manual_seed(7)
        q = torch.randn((1, 32, 128), generator=qg, device=dev).to(torch.bfloat16)
        for s in mine:
            torch.save(_attend_one(ops, pools[rank], s, k, v, q).cpu(), os.path.join(result_dir, f"b{s}.pt"))
        stats = sharding.migrate(moves, rank, pools, k, v, timeout_s=60.0)
        torch.cuda.synchronize(dev)
        dist.barrier()
        got = out1 if rank == 0 else out0
        ok = stats["device_ms"] is not None and stats["blocks_received"] == sum(
            (pools[rank].lens[s] + 15) // 16 for s in got)
        for s in got:
            after = _attend_one(ops, pools[rank], s, k, v, q).cpu()
            ok = ok and torch.equal(after, torch.load(os.path.join(result_dir, f"b{s}.pt")))
        ok = ok and ops.device_errors(rank) == 0
        with open(os.path.join(result_dir, f"ok{rank}"), "w") as f:
            f.write("1" if ok else "0")
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_migration_both_ways_over_nccl(cflib, tmp_path):
    """Six sequences, three each way, in one migrate() call: NCCL groups,
    deadline-bounded waits, attention bitwise unchanged on both ranks."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.start_processes(_worker_both_ways, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    assert (tmp_path / "ok0").read_text() == "1" and (tmp_path / "ok1").read_text() == "1"


def _worker_peer_gone(rank, world, port, result_dir):
    import datetime
    import time

    import torch
    import torch.distributed as dist

    from cacheflow_b200 import sharding

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20),
                            device_id=dev)
    dist.barrier()
    torch.cuda.synchronize(dev)
    if rank == 1:
        os._exit(0)  # leaves between steps, none of its kernels or collectives in flight
    ctx = np.array([3000, 700, 5000, 120], np.int64)
    pools = sharding.shard_workload(ctx, world, pool_factor=3.0, rng=np.random.default_rng(5))
    nb = max(p.num_blocks for p in pools)
    k = torch.zeros((nb, 8, 16, 128), dtype=torch.bfloat16, device=dev)
    v = torch.zeros_like(k)
    seq = max(pools[0].tables, key=lambda s: pools[0].lens[s])
    before = (dict(pools[0].tables), dict(pools[1].tables))
    t0 = time.monotonic()
    try:
        sharding.migrate([(seq, 0, 1)], 0, pools, k, v, timeout_s=3.0)
        res = "completed"
    except sharding.MigrationError as e:
        res = "error" if "did not arrive" in str(e) else "other"
    torch.cuda.synchronize(dev)  # nothing was posted: the device is idle
    unchanged = before == (dict(pools[0].tables), dict(pools[1].tables))
    with open(os.path.join(result_dir, "r0"), "w") as f:
        f.write(f"{res} {unchanged} {time.monotonic() - t0:.2f}")
    dist.distributed_c10d._abort_process_group()
    os._exit(0)


def test_migration_to_a_rank_that_left_over_nccl(cflib, tmp_path):
    """Rank 1 exits between steps; rank 0's migrate() learns it on the host
    (the process group's store) and raises MigrationError before posting any
    NCCL operation, its pools unchanged and its GPU idle (NVLS off)."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.start_processes(_worker_peer_gone, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    res, unchanged, secs = (tmp_path / "r0").read_text().split()
    assert res == "error" and unchanged == "True", (res, unchanged)
    assert float(secs) < 10.0
