"""CacheFlow's own C++ call shape on the GPU: cacheflow::cuda::launch_*
called through CacheFlow's UNCHANGED headers (paged_attention.cuh:44-54,
kv_cache_kernels.cuh:17-56, memory_utils.cuh:17-36) by a driver compiled
against them and linked to libcacheflow_b200.so (oracle/ref_api_driver.cpp).

The cache operators must be bit-identical to CacheFlow's own kernels on the
same inputs, including swap's (src, dst) argument order
(kv_cache_kernels.cu:121-131: the launcher hands the kernel (dst, src), so the
data flows src -> dst); attention through the reference signatures must be
within 1e-5 of the oracle (fp32, any context length), and within 1e-5 of
CacheFlow's own V1 kernel where that one is correct (contexts <= 128).
"""

import math

import numpy as np
import pytest

from cacheflow_b200.workloads import host_values
from helpers import as_f64, assert_close, random_tables, to_dev

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def api(cflib, oracle_mod):
    try:
        return oracle_mod.RefApi().lib
    except FileNotFoundError:
        pytest.skip("oracle/_ref/libcf_ref_api.so not built (make -C oracle ref)")


@pytest.fixture(scope="module")
def refk(oracle_mod):
    try:
        return oracle_mod.RefCuda().lib
    except FileNotFoundError:
        pytest.skip("oracle/_ref/libcf_ref_cuda.so not built (make -C oracle ref)")


def _stream():
    import torch

    return torch.cuda.current_stream().cuda_stream


def test_cache_operators_match_reference_kernels(api, refk):
    import torch

    rng = np.random.default_rng(91)
    pool, Hkv, D, T = 64, 4, 128, 50
    kc = to_dev(host_values((pool, Hkv, 16, D), "f32", 1.0, rng))
    vc = to_dev(host_values((pool, Hkv, 16, D), "f32", 1.0, rng))
    key = to_dev(host_values((T, Hkv, D), "f32", 1.0, rng))
    val = to_dev(host_values((T, Hkv, D), "f32", 1.0, rng))
    slots = to_dev(rng.permutation(pool * 16)[:T].astype(np.int32))
    a_k, a_v, b_k, b_v = kc.clone(), vc.clone(), kc.clone(), vc.clone()

    assert api.api_reshape_and_cache(key.data_ptr(), val.data_ptr(), a_k.data_ptr(), a_v.data_ptr(),
                                     slots.data_ptr(), T, Hkv, D, 16, _stream()) == 0
    torch.cuda.synchronize()
    assert refk.ref_reshape_and_cache(key.data_ptr(), val.data_ptr(), b_k.data_ptr(), b_v.data_ptr(),
                                      slots.data_ptr(), T, Hkv, D, 16) == 0
    assert torch.equal(a_k, b_k) and torch.equal(a_v, b_v)

    ids = rng.permutation(pool)
    pairs = to_dev(np.stack([ids[:10], ids[10:20]], 1).astype(np.int64))
    assert api.api_copy_blocks(a_k.data_ptr(), a_v.data_ptr(), pairs.data_ptr(), 10, Hkv, D, 16, _stream()) == 0
    torch.cuda.synchronize()
    assert refk.ref_copy_blocks(b_k.data_ptr(), b_v.data_ptr(), pairs.data_ptr(), 10, Hkv, D, 16) == 0
    assert torch.equal(a_k, b_k) and torch.equal(a_v, b_v)

    # swap out to pinned host memory and back in, CacheFlow's (src, dst) order
    blk = a_k[0].numel() * 4
    host_a = torch.zeros((24, Hkv, 16, D)).pin_memory()
    host_b = host_a.clone().pin_memory()
    out_map = to_dev(np.stack([ids[:8], np.arange(8) * 3], 1).astype(np.int64))
    assert api.api_swap_blocks(a_k.data_ptr(), host_a.data_ptr(), out_map.data_ptr(), 8, blk, _stream()) == 0
    torch.cuda.synchronize()
    assert refk.ref_swap_blocks(b_k.data_ptr(), host_b.data_ptr(), out_map.data_ptr(), 8, blk) == 0
    assert torch.equal(host_a, host_b)
    assert torch.equal(host_a[0], a_k[int(ids[0])].cpu())  # data went src -> dst
    in_map = to_dev(np.stack([np.arange(8) * 3, ids[30:38]], 1).astype(np.int64))
    assert api.api_swap_blocks(host_a.data_ptr(), a_v.data_ptr(), in_map.data_ptr(), 8, blk, _stream()) == 0
    torch.cuda.synchronize()
    assert refk.ref_swap_blocks(host_b.data_ptr(), b_v.data_ptr(), in_map.data_ptr(), 8, blk) == 0
    assert torch.equal(a_v, b_v)

    used = rng.random(pool) < 0.5
    from cacheflow_b200 import ops

    s, d = ops.compaction_plan(used)
    s_d, d_d = to_dev(s), to_dev(d)
    assert api.api_compact_kv_cache(a_k.data_ptr(), a_v.data_ptr(), s_d.data_ptr(), d_d.data_ptr(), len(s), Hkv,
                                    D, 16, _stream()) == 0
    torch.cuda.synchronize()
    assert refk.ref_compact_kv_cache(b_k.data_ptr(), b_v.data_ptr(), s_d.data_ptr(), d_d.data_ptr(), len(s), Hkv,
                                     D, 16) == 0
    assert torch.equal(a_k, b_k) and torch.equal(a_v, b_v)

    zero = to_dev(np.array([3, 0, 63], np.int32))
    assert api.api_memset_blocks(a_k.data_ptr(), zero.data_ptr(), 3, blk, _stream()) == 0
    torch.cuda.synchronize()
    assert refk.ref_memset_blocks(b_k.data_ptr(), zero.data_ptr(), 3, blk) == 0
    assert torch.equal(a_k, b_k)

    dst = torch.empty_like(a_v)
    assert api.api_async_memcpy_d2d(dst.data_ptr(), a_v.data_ptr(), a_v.numel() * 4, _stream()) == 0
    api.api_synchronize_device()
    assert torch.equal(dst, a_v)


@pytest.mark.parametrize("H,Hkv,D", [(8, 2, 128), (4, 4, 64), (16, 1, 128)])
def test_attention_through_reference_signatures(api, refk, oracle_mod, H, Hkv, D):
    import torch

    from cacheflow_b200 import ops

    rng = np.random.default_rng(92 + H + D)
    ctx = [1, 17, 128, 129, 600, 2000, 5]
    S = len(ctx)
    pool = sum((c + 15) // 16 for c in ctx) + 7
    tables = random_tables(rng, ctx, pool)
    q_h = host_values((S, H, D), "f32", 1.0, rng)
    k_h = host_values((pool, Hkv, 16, D), "f32", 1.0, rng)
    v_h = host_values((pool, Hkv, 16, D), "f32", 1.0, rng)
    q, k, v = to_dev(q_h), to_dev(k_h), to_dev(v_h)
    bt, cl = to_dev(tables), to_dev(np.array(ctx, np.int32))
    scale = 1.0 / math.sqrt(D)
    want = oracle_mod.paged_attention(q_h, k_h, v_h, tables, np.array(ctx, np.int32), scale)
    mb = tables.shape[1]

    out1 = torch.full((S, H, D), 5.0, device="cuda")
    assert api.api_paged_attention_v1(q.data_ptr(), k.data_ptr(), v.data_ptr(), out1.data_ptr(), bt.data_ptr(),
                                      cl.data_ptr(), scale, S, H, Hkv, D, 16, max(ctx), mb, _stream()) == 0
    P = ops.v2_num_partitions(max(ctx))
    es = torch.full((S, H, P), float("nan"), device="cuda")  # no pre-zeroing needed
    ml = torch.full_like(es, float("nan"))
    tmp = torch.full((S, H, P, D), float("nan"), device="cuda")
    out2 = torch.full((S, H, D), 5.0, device="cuda")
    assert api.api_paged_attention_v2(q.data_ptr(), k.data_ptr(), v.data_ptr(), out2.data_ptr(), bt.data_ptr(),
                                      cl.data_ptr(), scale, S, H, Hkv, D, 16, max(ctx), mb, es.data_ptr(),
                                      ml.data_ptr(), tmp.data_ptr(), P, _stream()) == 0
    torch.cuda.synchronize()
    assert ops.device_errors(0) == 0
    assert_close(as_f64(out1), want, "f32", "launch_paged_attention_v1 vs oracle")
    assert_close(as_f64(out2), want, "f32", "launch_paged_attention_v2 vs oracle")

    # CacheFlow's own V1 kernel, on the rows it computes correctly (<= 128 tokens)
    short = [i for i, c in enumerate(ctx) if c <= 128]
    qs, ts = to_dev(q_h[short]), to_dev(np.ascontiguousarray(tables[short]))
    cs = to_dev(np.array([ctx[i] for i in short], np.int32))
    ref_out = torch.zeros((len(short), H, D), device="cuda")
    assert refk.ref_paged_attention_v1(qs.data_ptr(), k.data_ptr(), v.data_ptr(), ref_out.data_ptr(), ts.data_ptr(),
                                       cs.data_ptr(), scale, len(short), H, Hkv, D, 16, 128, mb) == 0
    assert_close(as_f64(out1[short]), as_f64(ref_out), "f32", "ours vs CacheFlow's V1 kernel (contexts <= 128)")


def test_reference_signature_reports_unsupported_shape(api):
    """A shape the reference silently skipped (head_dim 96, paged_attention.cu:
    344-356) launches nothing here either, but last_status() says why."""
    import torch

    from cacheflow_b200 import _lib

    q = torch.zeros((1, 4, 96), device="cuda")
    kv = torch.zeros((2, 4, 16, 96), device="cuda")
    out = torch.full((1, 4, 96), 3.0, device="cuda")
    bt = to_dev(np.array([[0]], np.int32))
    cl = to_dev(np.array([5], np.int32))
    st = api.api_paged_attention_v1(q.data_ptr(), kv.data_ptr(), kv.data_ptr(), out.data_ptr(), bt.data_ptr(),
                                    cl.data_ptr(), 0.1, 1, 4, 4, 96, 16, 5, 1, _stream())
    torch.cuda.synchronize()
    assert st == _lib.CF_ERR_UNSUPPORTED
    assert torch.equal(out, torch.full_like(out, 3.0))
