"""Bit-exact parity of the KV-cache data-movement kernels with the CPU oracle
(and with CacheFlow's own CUDA kernels, built from its sources into
oracle/_ref, when that library is present), through the C ABI."""

import numpy as np
import pytest

from cacheflow_b200.workloads import host_values
from helpers import random_tables, to_dev, to_host, torch_dtype

pytestmark = pytest.mark.gpu

DTYPES = ["f32", "f16", "bf16"]


def _cache(rng, dtype, pool, Hkv, D):
    return host_values((pool, Hkv, 16, D), dtype, 1.0, rng)


def _ref_cuda(oracle_mod):
    try:
        return oracle_mod.RefCuda()
    except FileNotFoundError:
        return None


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("Hkv,D", [(8, 128), (2, 64), (1, 256)])
def test_reshape_and_cache_bit_exact(cflib, oracle_mod, dtype, Hkv, D):
    from cacheflow_b200 import ops

    rng = np.random.default_rng(21)
    pool, T = 64, 200
    kc, vc = _cache(rng, dtype, pool, Hkv, D), _cache(rng, dtype, pool, Hkv, D)
    key, val = host_values((T, Hkv, D), dtype, 1.0, rng), host_values((T, Hkv, D), dtype, 1.0, rng)
    # distinct slots, including the first and the last slot of the pool
    slots = np.concatenate([[0, pool * 16 - 1], 1 + rng.permutation(pool * 16 - 2)[: T - 2]]).astype(np.int32)
    slots[5] = -1  # padding token: skipped
    dk, dv = to_dev(kc, dtype), to_dev(vc, dtype)
    ops.reshape_and_cache(to_dev(key, dtype), to_dev(val, dtype), dk, dv, to_dev(slots))
    oracle_mod.reshape_and_cache(key, val, kc, vc, slots)
    assert np.array_equal(to_host(dk), kc) and np.array_equal(to_host(dv), vc)
    assert ops.device_errors(0) == 0


def test_reshape_and_cache_bad_slot_recorded(cflib):
    from cacheflow_b200 import _lib, ops

    rng = np.random.default_rng(22)
    kc = to_dev(_cache(rng, "bf16", 4, 2, 128), "bf16")
    vc = kc.clone()
    before = kc.clone()
    key = to_dev(host_values((2, 2, 128), "bf16", 1.0, rng), "bf16")
    ops.device_errors(0, clear=True)
    ops.reshape_and_cache(key, key, kc, vc, to_dev(np.array([4 * 16, 10**6], np.int32)))
    assert ops.device_errors(0, clear=True) & _lib.CF_DEVERR_SLOT
    import torch

    assert torch.equal(kc, before)


@pytest.mark.parametrize("dtype", DTYPES)
def test_copy_blocks_bit_exact(cflib, oracle_mod, dtype):
    from cacheflow_b200 import ops

    rng = np.random.default_rng(23)
    pool, Hkv, D = 50, 8, 128
    kc, vc = _cache(rng, dtype, pool, Hkv, D), _cache(rng, dtype, pool, Hkv, D)
    ids = rng.permutation(pool)
    pairs = np.stack([ids[:16], ids[16:32]], 1).astype(np.int64)  # disjoint src / dst
    dk, dv = to_dev(kc, dtype), to_dev(vc, dtype)
    ops.copy_blocks(dk, dv, to_dev(pairs))
    oracle_mod.copy_blocks(kc, vc, pairs)
    assert np.array_equal(to_host(dk), kc) and np.array_equal(to_host(dv), vc)


@pytest.mark.parametrize("dtype", DTYPES)
def test_swap_blocks_device_host_round_trip(cflib, oracle_mod, dtype):
    import torch

    from cacheflow_b200 import ops

    rng = np.random.default_rng(24)
    pool, cpu_pool, Hkv, D = 40, 30, 4, 128
    gpu = _cache(rng, dtype, pool, Hkv, D)
    host = _cache(rng, dtype, cpu_pool, Hkv, D)
    dg = to_dev(gpu, dtype)
    dh = to_dev(host, dtype, device="cpu").pin_memory()
    out_pairs = np.stack([rng.permutation(pool)[:12], rng.permutation(cpu_pool)[:12]], 1).astype(np.int64)
    in_pairs = np.stack([out_pairs[:, 1], rng.permutation(pool)[:12]], 1).astype(np.int64)
    # device -> host (mapping read by the kernel from device memory)
    ops.swap_blocks(dg, dh, to_dev(out_pairs), stream_tensor=dg)
    torch.cuda.synchronize()
    oracle_mod.swap_blocks(gpu, host, out_pairs)
    assert np.array_equal(to_host(dh), host)
    # host -> device (mapping in pinned host memory)
    ops.swap_blocks(dh, dg, torch.from_numpy(in_pairs).pin_memory(), stream_tensor=dg)
    torch.cuda.synchronize()
    oracle_mod.swap_blocks(host, gpu, in_pairs)
    assert np.array_equal(to_host(dg), gpu)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_swap_blocks_dma_matches(cflib, oracle_mod, dtype):
    import torch

    from cacheflow_b200 import ops

    rng = np.random.default_rng(25)
    pool, cpu_pool, Hkv, D = 64, 64, 2, 128
    gpu = _cache(rng, dtype, pool, Hkv, D)
    host = _cache(rng, dtype, cpu_pool, Hkv, D)
    dg = to_dev(gpu, dtype)
    dh = to_dev(host, dtype, device="cpu").pin_memory()
    runs = np.concatenate([np.arange(5, 15), [40, 2, 3], np.arange(50, 60)])
    dst = np.concatenate([np.arange(20, 30), [7, 8, 9], np.arange(30, 40)])
    pairs = np.stack([runs, dst], 1).astype(np.int64)
    ops.swap_blocks_dma(dg, dh, pairs, stream_tensor=dg)
    torch.cuda.synchronize()
    oracle_mod.swap_blocks(gpu, host, pairs)
    assert np.array_equal(to_host(dh), host)


@pytest.mark.parametrize("dtype", DTYPES)
def test_compact_kv_cache_bit_exact(cflib, oracle_mod, dtype):
    from cacheflow_b200 import _lib, ops

    rng = np.random.default_rng(26)
    pool, Hkv, D = 300, 8, 128
    kc, vc = _cache(rng, dtype, pool, Hkv, D), _cache(rng, dtype, pool, Hkv, D)
    used = rng.random(pool) < 0.5
    src, dst = ops.compaction_plan(used)
    assert ops.check_compaction_plan(src, dst, pool) == _lib.CF_OK
    # an identity move is skipped like in the reference
    src = np.append(src, 3).astype(np.int32)
    dst = np.append(dst, 3).astype(np.int32)
    dk, dv = to_dev(kc, dtype), to_dev(vc, dtype)
    ops.compact_kv_cache(dk, dv, to_dev(src), to_dev(dst))
    oracle_mod.compact_kv_cache(kc, vc, src, dst)
    assert np.array_equal(to_host(dk), kc) and np.array_equal(to_host(dv), vc)


def test_memset_blocks(cflib, oracle_mod):
    from cacheflow_b200 import ops

    rng = np.random.default_rng(27)
    c = _cache(rng, "f32", 20, 4, 128)
    ids = np.array([0, 7, 19], np.int32)
    d = to_dev(c, "f32")
    ops.memset_blocks(d, to_dev(ids))
    oracle_mod.memset_blocks(c, ids)
    assert np.array_equal(to_host(d), c)


def test_against_reference_cuda_kernels(cflib, oracle_mod):
    """Same fp32 inputs through CacheFlow's own kernels and ours: bit-identical."""
    import torch

    from cacheflow_b200 import ops

    ref = _ref_cuda(oracle_mod)
    if ref is None:
        pytest.skip("oracle/_ref/libcf_ref_cuda.so not built")
    L = ref.lib
    rng = np.random.default_rng(28)
    pool, Hkv, D, T = 64, 4, 128, 50
    kc = to_dev(_cache(rng, "f32", pool, Hkv, D))
    vc = to_dev(_cache(rng, "f32", pool, Hkv, D))
    key = to_dev(host_values((T, Hkv, D), "f32", 1.0, rng))
    val = to_dev(host_values((T, Hkv, D), "f32", 1.0, rng))
    slots = to_dev(rng.permutation(pool * 16)[:T].astype(np.int32))
    a_k, a_v, b_k, b_v = kc.clone(), vc.clone(), kc.clone(), vc.clone()
    ops.reshape_and_cache(key, val, a_k, a_v, slots)
    torch.cuda.synchronize()
    assert L.ref_reshape_and_cache(key.data_ptr(), val.data_ptr(), b_k.data_ptr(), b_v.data_ptr(),
                                   slots.data_ptr(), T, Hkv, D, 16) == 0
    assert torch.equal(a_k, b_k) and torch.equal(a_v, b_v)

    ids = rng.permutation(pool)
    pairs = to_dev(np.stack([ids[:10], ids[10:20]], 1).astype(np.int64))
    ops.copy_blocks(a_k, a_v, pairs)
    torch.cuda.synchronize()
    assert L.ref_copy_blocks(b_k.data_ptr(), b_v.data_ptr(), pairs.data_ptr(), 10, Hkv, D, 16) == 0
    assert torch.equal(a_k, b_k) and torch.equal(a_v, b_v)

    used = rng.random(pool) < 0.5
    s, d = ops.compaction_plan(used)
    s_d, d_d = to_dev(s), to_dev(d)
    ops.compact_kv_cache(a_k, a_v, s_d, d_d)
    torch.cuda.synchronize()
    assert L.ref_compact_kv_cache(b_k.data_ptr(), b_v.data_ptr(), s_d.data_ptr(), d_d.data_ptr(),
                                  len(s), Hkv, D, 16) == 0
    assert torch.equal(a_k, b_k) and torch.equal(a_v, b_v)

    blk = a_k[0].numel() * 4
    dst_a = torch.zeros((30, Hkv, 16, D), device="cuda")
    dst_b = dst_a.clone()
    sp = to_dev(np.stack([ids[:8], np.arange(8) * 3], 1).astype(np.int64))
    ops.swap_blocks(a_k, dst_a, sp)
    torch.cuda.synchronize()
    assert L.ref_swap_blocks(b_k.data_ptr(), dst_b.data_ptr(), sp.data_ptr(), 8, blk) == 0
    assert torch.equal(dst_a, dst_b)

    mids = to_dev(np.array([1, 5, 9], np.int32))
    ops.memset_blocks(a_v, mids)
    torch.cuda.synchronize()
    assert L.ref_memset_blocks(b_v.data_ptr(), mids.data_ptr(), 3, blk) == 0
    assert torch.equal(a_v, b_v)


def test_reference_v1_short_contexts_agree(cflib, oracle_mod):
    """Where CacheFlow's V1 kernel is correct (ctx <= 128, D 128/64), it agrees
    with ours and with the oracle within the fp32 tolerance."""
    import math

    import torch

    from cacheflow_b200 import ops
    from helpers import as_f64, assert_close

    ref = _ref_cuda(oracle_mod)
    if ref is None:
        pytest.skip("oracle/_ref/libcf_ref_cuda.so not built")
    rng = np.random.default_rng(29)
    for D, H, Hkv in [(128, 4, 4), (64, 8, 2)]:
        ctx = [1, 15, 16, 17, 64, 128]
        pool = sum((c + 15) // 16 for c in ctx) + 3
        tables = random_tables(rng, ctx, pool)
        q = host_values((len(ctx), H, D), "f32", 1.0, rng)
        k = host_values((pool, Hkv, 16, D), "f32", 1.0, rng)
        v = host_values((pool, Hkv, 16, D), "f32", 1.0, rng)
        dq, dk, dv, bt = to_dev(q), to_dev(k), to_dev(v), to_dev(tables)
        cl = to_dev(np.array(ctx, np.int32))
        ours = torch.empty_like(dq)
        theirs = torch.empty_like(dq)
        scale = 1.0 / math.sqrt(D)
        ops.paged_attention_v1(ours, dq, dk, dv, bt, cl, scale, max(ctx))
        torch.cuda.synchronize()
        assert ref.lib.ref_paged_attention_v1(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), theirs.data_ptr(),
                                              bt.data_ptr(), cl.data_ptr(), scale, len(ctx), H, Hkv, D, 16,
                                              max(ctx), tables.shape[1]) == 0
        want = oracle_mod.paged_attention(q, k, v, tables, np.array(ctx, np.int32), scale)
        assert_close(as_f64(theirs), want, "f32", "reference V1 vs oracle")
        assert_close(as_f64(ours), want, "f32", "ours vs oracle")


def test_execute_block_ops_matches_sequential_application(cflib):
    """One step's scheduler block ops (swap-outs, swap-ins, then COW copies,
    for K and V) equal applying the lists in that order on the host."""
    import torch

    from cacheflow_b200 import ops

    rng = np.random.default_rng(31)
    ngpu, ncpu, shape = 24, 16, (8, 16, 64)
    gk = torch.from_numpy(rng.standard_normal((ngpu,) + shape).astype(np.float32)).to(torch.bfloat16)
    gv = torch.from_numpy(rng.standard_normal((ngpu,) + shape).astype(np.float32)).to(torch.bfloat16)
    ck = torch.from_numpy(rng.standard_normal((ncpu,) + shape).astype(np.float32)).to(torch.bfloat16).pin_memory()
    cv = torch.from_numpy(rng.standard_normal((ncpu,) + shape).astype(np.float32)).to(torch.bfloat16).pin_memory()
    # swap-outs include a run of consecutive ids (one merged copy)
    swaps_out = np.array([[3, 0], [4, 1], [5, 2], [10, 7]], np.int64)
    swaps_in = np.array([[9, 3], [12, 20]], np.int64)       # GPU block 3 reused after its swap-out
    copies = np.array([[20, 21], [0, 5], [7, 8]], np.int64)  # copies see the swapped-in block 20
    want = [t.clone() for t in (gk, gv, ck, cv)]
    for src, dst in swaps_out:
        want[2][dst] = want[0][src]
        want[3][dst] = want[1][src]
    for src, dst in swaps_in:
        want[0][dst] = want[2][src]
        want[1][dst] = want[3][src]
    for src, dst in copies:
        want[0][dst] = want[0][src]
        want[1][dst] = want[1][src]
    dk, dv = gk.cuda(), gv.cuda()
    ops.execute_block_ops(dk, dv, ck, cv, swaps_out, swaps_in, copies)
    torch.cuda.synchronize()
    assert torch.equal(dk.cpu(), want[0]) and torch.equal(dv.cpu(), want[1])
    assert torch.equal(ck, want[2]) and torch.equal(cv, want[3])
    with pytest.raises(ops.CacheFlowError):  # a CPU id past the pool: nothing is enqueued
        ops.execute_block_ops(dk, dv, ck, cv, swaps_out=np.array([[0, ncpu]], np.int64))


def _apply_host(want, swaps_out, swaps_in, copies):
    for src, dst in swaps_out:
        want[2][dst] = want[0][src]
        want[3][dst] = want[1][src]
    for src, dst in swaps_in:
        want[0][dst] = want[2][src]
        want[1][dst] = want[3][src]
    for src, dst in copies:
        want[0][dst] = want[0][src]
        want[1][dst] = want[1][src]


@pytest.mark.parametrize("case", ["many_scattered", "long_runs", "chained_copies", "pageable_cpu_pool"])
def test_execute_block_ops_kernel_and_copy_engine_paths(cflib, case):
    """Every route of cf_execute_block_ops gives the sequential result:
    more than one kernel launch's worth of scattered pairs (4000 per launch),
    lists of long consecutive runs (copy engines), COW copies that form a
    chain (a destination read by a later pair: copy engines, in order), and a
    pageable CPU pool the kernel cannot address (copy engines)."""
    import torch

    from cacheflow_b200 import ops

    rng = np.random.default_rng({"many_scattered": 41, "long_runs": 42, "chained_copies": 43,
                                 "pageable_cpu_pool": 44}[case])
    ngpu, ncpu, shape = 12000, 9000, (2, 16, 8)  # 512-byte bf16 blocks
    if case != "many_scattered":
        ngpu, ncpu = 600, 400
    gk = torch.from_numpy(rng.standard_normal((ngpu,) + shape).astype(np.float32)).to(torch.bfloat16)
    gv = torch.from_numpy(rng.standard_normal((ngpu,) + shape).astype(np.float32)).to(torch.bfloat16)
    ck = torch.from_numpy(rng.standard_normal((ncpu,) + shape).astype(np.float32)).to(torch.bfloat16)
    cv = torch.from_numpy(rng.standard_normal((ncpu,) + shape).astype(np.float32)).to(torch.bfloat16)
    if case != "pageable_cpu_pool":
        ck, cv = ck.pin_memory(), cv.pin_memory()
    if case == "many_scattered":
        g = rng.permutation(ngpu)
        swaps_out = np.stack([g[:8500], rng.permutation(ncpu)[:8500]], 1)
        swaps_in = np.stack([rng.permutation(ncpu)[:4100], g[:4100]], 1)  # reuse swapped-out GPU blocks
        copies = np.stack([g[8500:8600], g[8600:8700]], 1)
    elif case == "long_runs":
        swaps_out = np.stack([np.arange(100, 300), np.arange(50, 250)], 1)
        swaps_in = np.stack([np.arange(0, 64), np.arange(100, 164)], 1)
        copies = np.stack([np.arange(400, 480), np.arange(500, 580)], 1)
    elif case == "chained_copies":
        swaps_out = np.stack([rng.permutation(ngpu)[:20], rng.permutation(ncpu)[:20]], 1)
        swaps_in = np.zeros((0, 2), np.int64)
        copies = np.array([[1, 2], [2, 3], [3, 4], [9, 7], [7, 11]], np.int64)  # 2..4 all become block 1
    else:
        swaps_out = np.stack([rng.permutation(ngpu)[:50], rng.permutation(ncpu)[:50]], 1)
        swaps_in = np.stack([rng.permutation(ncpu)[:30], rng.permutation(ngpu)[:30]], 1)
        copies = np.zeros((0, 2), np.int64)
    swaps_out, swaps_in, copies = (np.ascontiguousarray(x, np.int64) for x in (swaps_out, swaps_in, copies))
    want = [t.clone() for t in (gk, gv, ck, cv)]
    _apply_host(want, swaps_out, swaps_in, copies)
    dk, dv = gk.cuda(), gv.cuda()
    ops.execute_block_ops(dk, dv, ck, cv, swaps_out, swaps_in, copies)
    torch.cuda.synchronize()
    assert ops.device_errors(0) == 0
    assert torch.equal(dk.cpu(), want[0]) and torch.equal(dv.cpu(), want[1])
    assert torch.equal(ck, want[2]) and torch.equal(cv, want[3])
