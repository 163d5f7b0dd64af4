"""FP8 (e4m3) KV caches: the quantizing scatter (cf_reshape_and_cache_fp8) is
bit-exact against the oracle's rounding, decode attention over fp8 caches
(cf_paged_attention_fp8_v1/_v2, FMA and tensor-core consumers) matches the
oracle's attention over the dequantized caches within the 16-bit tolerance,
and the fused fp8 decode step (cf_paged_attention_fp8_append_v1/_v2) equals
the scatter followed by the attention bit for bit."""

import math

import numpy as np
import pytest

from cacheflow_b200.workloads import host_values
from helpers import CODE, as_f64, assert_close, random_tables, to_dev, torch_dtype

pytestmark = pytest.mark.gpu

K_SCALE, V_SCALE = 0.05, 0.1


def _fp8_cache(rng, shape):
    """Random e4m3 codes from N(0, 1) values (no NaN codes)."""
    import torch

    x = torch.from_numpy(rng.standard_normal(shape).astype(np.float32) * 2)
    return x.to(torch.float8_e4m3fn).view(torch.uint8).numpy()


def _to_fp8_dev(codes):
    import torch

    return torch.from_numpy(np.ascontiguousarray(codes)).cuda().view(torch.float8_e4m3fn)


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
def test_reshape_and_cache_fp8_bit_exact(cflib, oracle_mod, dtype):
    import torch

    from cacheflow_b200 import ops
    from helpers import to_host

    rng = np.random.default_rng(12)
    T, Hkv, D, pool = 300, 8, 128, 64
    key = host_values((T, Hkv, D), dtype, 20.0, rng)   # reaches past 448 * scale: saturation
    val = host_values((T, Hkv, D), dtype, 0.02, rng)   # small: subnormal codes
    slots = rng.permutation(pool * 16)[:T].astype(np.int32)
    slots[::37] = -1
    kc = np.zeros((pool, Hkv, 16, D), np.uint8)
    vc = np.zeros_like(kc)
    dk, dv = _to_fp8_dev(kc), _to_fp8_dev(vc)
    ops.reshape_and_cache_fp8(to_dev(key, dtype), to_dev(val, dtype), dk, dv, to_dev(slots), K_SCALE, V_SCALE)
    oracle_mod.reshape_and_cache_fp8(key, val, kc, vc, slots, K_SCALE, V_SCALE, CODE[dtype])
    assert np.array_equal(dk.view(torch.uint8).cpu().numpy(), kc)
    assert np.array_equal(dv.view(torch.uint8).cpu().numpy(), vc)
    assert ops.device_errors(0) == 0


CASES = [
    # query dtype, num_heads, num_kv_heads, head_dim, contexts
    ("f16", 8, 8, 128, [1, 15, 16, 17, 129, 512, 513, 3000]),
    ("bf16", 32, 8, 128, [1, 16, 17, 700, 1025, 9000]),   # group 4: tensor-core consumer
    ("bf16", 32, 2, 128, [3, 160, 1030]),                 # group 16: two head chunks
    ("f16", 8, 4, 128, [5, 300]),                         # group 2
    ("bf16", 8, 8, 256, [1, 17, 300]),
    ("f16", 16, 2, 256, [1, 100, 1500]),
]


@pytest.fixture(params=["auto", "fma", "mma"])
def consumer(request, monkeypatch):
    if request.param == "auto":
        monkeypatch.delenv("CF_ATTN_CONSUMER", raising=False)
    else:
        monkeypatch.setenv("CF_ATTN_CONSUMER", request.param)
    return request.param


@pytest.mark.parametrize("path", ["v1", "v1_split", "v2"])
@pytest.mark.parametrize("dtype,H,Hkv,D,ctx", CASES)
def test_fp8_attention_matches_oracle(cflib, oracle_mod, consumer, path, dtype, H, Hkv, D, ctx):
    import torch

    from cacheflow_b200 import ops

    rng = np.random.default_rng(hash((dtype, H, Hkv, D, len(ctx), path)) % 2**32)
    S = len(ctx)
    pool = sum((c + 15) // 16 for c in ctx) + 5
    tables = random_tables(rng, ctx, pool)
    cl = np.array(ctx, np.int32)
    q = host_values((S, H, D), dtype, 0.5, rng)
    kc, vc = _fp8_cache(rng, (pool, Hkv, 16, D)), _fp8_cache(rng, (pool, Hkv, 16, D))
    dq, dk, dv = to_dev(q, dtype), _to_fp8_dev(kc), _to_fp8_dev(vc)
    bt, dcl = to_dev(tables), to_dev(cl)
    out = torch.full((S, H, D), 5.0, dtype=torch_dtype(dtype), device="cuda")
    mctx = int(cl.max())
    if path == "v2":
        P = ops.v2_num_partitions(mctx)
        es = torch.empty((S, H, P), device="cuda")
        ml = torch.empty_like(es)
        to = torch.empty((S, H, P, D), device="cuda")
        ops.paged_attention_fp8_v2(out, es, ml, to, dq, dk, dv, bt, dcl, K_SCALE, V_SCALE)
    else:
        ws = None
        if path == "v1_split":
            n = ops.paged_attention_v1_workspace_size(dq, dk, bt, mctx)
            ws = torch.empty(max(n, 16), dtype=torch.uint8, device="cuda") if n else None
        ops.paged_attention_fp8_v1(out, dq, dk, dv, bt, dcl, K_SCALE, V_SCALE, workspace=ws)
    want = oracle_mod.paged_attention_fp8(q, kc, vc, tables, cl, 1 / math.sqrt(D), K_SCALE, V_SCALE, CODE[dtype],
                                          num_threads=8)
    assert_close(as_f64(out), want, dtype, f"fp8 attention {path}")
    assert ops.device_errors(0) == 0


APPEND_CASES = [
    ("f16", 8, 8, 128, [1, 15, 16, 17, 513, 3000]),
    ("bf16", 32, 8, 128, [1, 2, 16, 17, 1025, 4000]),
    ("bf16", 32, 2, 128, [3, 160, 1030]),
    ("f16", 16, 2, 256, [1, 17, 1500]),
]


@pytest.mark.parametrize("path", ["v1", "v1_split", "v2"])
@pytest.mark.parametrize("dtype,H,Hkv,D,ctx", APPEND_CASES)
def test_fp8_append_equals_reshape_then_attention(cflib, oracle_mod, consumer, path, dtype, H, Hkv, D, ctx):
    """cf_paged_attention_fp8_append_v1/_v2 store the same e4m3 bytes as
    cf_reshape_and_cache_fp8 and return the same output, bit for bit, as
    that scatter followed by cf_paged_attention_fp8_v1/_v2."""
    import torch

    from cacheflow_b200 import ops

    rng = np.random.default_rng(hash(("fp8_append", dtype, H, Hkv, D, len(ctx), path)) % 2**32)
    S = len(ctx)
    pool = sum((c + 15) // 16 for c in ctx) + 5
    tables = random_tables(rng, ctx, pool)
    cl = np.array(ctx, np.int32)
    pos = cl - 1
    slots = (tables[np.arange(S), pos // 16] * 16 + pos % 16).astype(np.int32)
    q = host_values((S, H, D), dtype, 0.5, rng)
    nk = host_values((S, Hkv, D), dtype, 20.0, rng)    # past 448 * K_SCALE: saturates
    nv = host_values((S, Hkv, D), dtype, 0.02, rng)    # subnormal codes
    kc, vc = _fp8_cache(rng, (pool, Hkv, 16, D)), _fp8_cache(rng, (pool, Hkv, 16, D))
    dq, dnk, dnv = to_dev(q, dtype), to_dev(nk, dtype), to_dev(nv, dtype)
    bt, dcl, dsl = to_dev(tables), to_dev(cl), to_dev(slots)
    mctx = int(cl.max())

    def run(fused, with_slots):
        dk, dv = _to_fp8_dev(kc), _to_fp8_dev(vc)
        out = torch.full((S, H, D), 3.0, dtype=torch_dtype(dtype), device="cuda")
        sl = dsl if with_slots else None
        if not fused:
            ops.reshape_and_cache_fp8(dnk, dnv, dk, dv, dsl, K_SCALE, V_SCALE)
        if path == "v2":
            P = ops.v2_num_partitions(mctx)
            es = torch.empty((S, H, P), device="cuda")
            ml = torch.empty_like(es)
            to = torch.empty((S, H, P, D), device="cuda")
            if fused:
                ops.paged_attention_fp8_append_v2(out, es, ml, to, dq, dnk, dnv, dk, dv, bt, dcl, K_SCALE, V_SCALE,
                                                  sl)
            else:
                ops.paged_attention_fp8_v2(out, es, ml, to, dq, dk, dv, bt, dcl, K_SCALE, V_SCALE)
        else:
            ws = None
            if path == "v1_split":
                n = ops.paged_attention_v1_workspace_size(dq, dk, bt, mctx)
                ws = torch.empty(max(n, 16), dtype=torch.uint8, device="cuda") if n else None
            if fused:
                ops.paged_attention_fp8_append_v1(out, dq, dnk, dnv, dk, dv, bt, dcl, K_SCALE, V_SCALE, sl,
                                                  workspace=ws)
            else:
                ops.paged_attention_fp8_v1(out, dq, dk, dv, bt, dcl, K_SCALE, V_SCALE, workspace=ws)
        return out, dk.view(torch.uint8), dv.view(torch.uint8)

    ops.device_errors(0, clear=True)
    o_ref, k_ref, v_ref = run(False, True)
    for with_slots in (False, True):
        o, kk, vv = run(True, with_slots)
        assert torch.equal(kk, k_ref) and torch.equal(vv, v_ref), "fp8 cache after the fused append"
        assert torch.equal(o, o_ref), "fused fp8 output differs from reshape_and_cache_fp8 + attention"
    assert ops.device_errors(0) == 0
    k2, v2 = kc.copy(), vc.copy()
    oracle_mod.reshape_and_cache_fp8(nk, nv, k2, v2, slots, K_SCALE, V_SCALE, CODE[dtype])
    assert np.array_equal(k_ref.cpu().numpy(), k2) and np.array_equal(v_ref.cpu().numpy(), v2)
    want = oracle_mod.paged_attention_fp8(q, k2, v2, tables, cl, 1 / math.sqrt(D), K_SCALE, V_SCALE, CODE[dtype],
                                          num_threads=8)
    assert_close(as_f64(o_ref), want, dtype, f"fp8 append {path}")


def test_fp8_append_wrong_slot_appends_nothing(cflib, oracle_mod):
    import torch

    from cacheflow_b200 import _lib, ops

    rng = np.random.default_rng(16)
    ctx = [20, 33, 700, 64]
    tables = random_tables(rng, ctx, 60)
    cl = np.array(ctx, np.int32)
    pos = cl - 1
    slots = (tables[np.arange(4), pos // 16] * 16 + pos % 16).astype(np.int32)
    bad = slots.copy()
    bad[1] = -1
    bad[2] = slots[2] + 1
    q = host_values((4, 32, 128), "bf16", 0.5, rng)
    nk = host_values((4, 8, 128), "bf16", 0.5, rng)
    nv = host_values((4, 8, 128), "bf16", 0.5, rng)
    kc, vc = _fp8_cache(rng, (60, 8, 16, 128)), _fp8_cache(rng, (60, 8, 16, 128))
    dk, dv = _to_fp8_dev(kc), _to_fp8_dev(vc)
    out = torch.empty((4, 32, 128), dtype=torch.bfloat16, device="cuda")
    ops.device_errors(0, clear=True)
    ops.paged_attention_fp8_append_v1(out, to_dev(q, "bf16"), to_dev(nk, "bf16"), to_dev(nv, "bf16"), dk, dv,
                                      to_dev(tables), to_dev(cl), K_SCALE, V_SCALE, to_dev(bad))
    assert ops.device_errors(0, clear=True) == _lib.CF_DEVERR_SLOT
    ok = np.array([True, False, False, True])
    k2, v2 = kc.copy(), vc.copy()
    oracle_mod.reshape_and_cache_fp8(nk[ok], nv[ok], k2, v2, slots[ok], K_SCALE, V_SCALE, CODE["bf16"])
    assert np.array_equal(dk.view(torch.uint8).cpu().numpy(), k2)
    assert np.array_equal(dv.view(torch.uint8).cpu().numpy(), v2)
    want = oracle_mod.paged_attention_fp8(q, k2, v2, tables, cl, 1 / math.sqrt(128), K_SCALE, V_SCALE, CODE["bf16"])
    assert_close(as_f64(out), want, "bf16", "rows that append nothing attend to the cache as it is")


@pytest.mark.parametrize("path", ["v1", "v2"])
def test_fp8_attention_wide_score_range(cflib, oracle_mod, path):
    """Scores spanning ~40 (log2 units) in random block order: the running
    reference point both moves (by more than the lazy threshold) and stays
    put while blocks below it are added."""
    import torch

    from cacheflow_b200 import ops

    rng = np.random.default_rng(17)
    ctx = [3000, 700, 16, 5000]
    S, H, Hkv, D = len(ctx), 32, 8, 128
    pool = sum((c + 15) // 16 for c in ctx) + 3
    tables = random_tables(rng, ctx, pool)
    cl = np.array(ctx, np.int32)
    q = host_values((S, H, D), "bf16", 0.5, rng)
    ramp = (0.05 + 4.0 * rng.random(pool) ** 2).astype(np.float32)[:, None, None, None]
    x = torch.from_numpy(rng.standard_normal((pool, Hkv, 16, D)).astype(np.float32) * 2 * ramp)
    kc = x.to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    vc = _fp8_cache(rng, (pool, Hkv, 16, D))
    ks, vs = 1.0, 0.1
    dq, dk, dv = to_dev(q, "bf16"), _to_fp8_dev(kc), _to_fp8_dev(vc)
    bt, dcl = to_dev(tables), to_dev(cl)
    out = torch.empty((S, H, D), dtype=torch.bfloat16, device="cuda")
    if path == "v2":
        P = ops.v2_num_partitions(int(cl.max()))
        es = torch.empty((S, H, P), device="cuda")
        ml = torch.empty_like(es)
        to = torch.empty((S, H, P, D), device="cuda")
        ops.paged_attention_fp8_v2(out, es, ml, to, dq, dk, dv, bt, dcl, ks, vs)
    else:
        ops.paged_attention_fp8_v1(out, dq, dk, dv, bt, dcl, ks, vs)
    want = oracle_mod.paged_attention_fp8(q, kc, vc, tables, cl, 1 / math.sqrt(D), ks, vs, CODE["bf16"],
                                          num_threads=8)
    assert_close(as_f64(out), want, "bf16", f"fp8 attention, wide score range, {path}")
    assert ops.device_errors(0) == 0


def test_fp8_nan_codes_past_context_do_not_leak(cflib, oracle_mod, consumer):
    import torch

    from cacheflow_b200 import ops

    rng = np.random.default_rng(14)
    ctx = [20, 33, 7]
    tables = random_tables(rng, ctx, 12)
    cl = np.array(ctx, np.int32)
    q = host_values((3, 32, 128), "bf16", 0.5, rng)
    kc, vc = _fp8_cache(rng, (12, 8, 16, 128)), _fp8_cache(rng, (12, 8, 16, 128))
    for s, c in enumerate(ctx):
        b = tables[s][c // 16]
        kc[b, :, c % 16:] = 0x7F   # e4m3 NaN
        vc[b, :, c % 16:] = 0xFF
    out = torch.empty((3, 32, 128), dtype=torch.bfloat16, device="cuda")
    ops.paged_attention_fp8_v1(out, to_dev(q, "bf16"), _to_fp8_dev(kc), _to_fp8_dev(vc), to_dev(tables),
                               to_dev(cl), K_SCALE, V_SCALE)
    want = oracle_mod.paged_attention_fp8(q, kc, vc, tables, cl, 1 / math.sqrt(128), K_SCALE, V_SCALE, CODE["bf16"])
    assert_close(as_f64(out), want, "bf16", "fp8 with NaN codes past the context")


def test_fp8_caches_move_as_bytes(cflib):
    import torch

    from cacheflow_b200 import ops

    rng = np.random.default_rng(15)
    kc = _to_fp8_dev(_fp8_cache(rng, (20, 8, 16, 128)))
    vc = _to_fp8_dev(_fp8_cache(rng, (20, 8, 16, 128)))
    k0, v0 = kc.view(torch.uint8).clone(), vc.view(torch.uint8).clone()
    pairs = torch.tensor([[1, 5], [7, 2]], dtype=torch.int64, device="cuda")
    ops.copy_blocks(kc, vc, pairs)
    ku = kc.view(torch.uint8)
    assert torch.equal(ku[5], k0[1]) and torch.equal(ku[2], k0[7]) and torch.equal(ku[0], k0[0])
    ops.memset_blocks(kc, torch.tensor([3], dtype=torch.int32, device="cuda"))
    assert int(kc.view(torch.uint8)[3].count_nonzero()) == 0
    ops.compact_kv_cache(kc, vc, torch.tensor([9], dtype=torch.int32, device="cuda"),
                         torch.tensor([4], dtype=torch.int32, device="cuda"))
    assert torch.equal(vc.view(torch.uint8)[4], v0[9])


def test_fp8_rejects_unsupported(cflib):
    import torch

    from cacheflow_b200 import _lib, ops

    q = torch.zeros((1, 8, 64), dtype=torch.float16, device="cuda")
    kc = torch.zeros((2, 8, 16, 64), dtype=torch.float8_e4m3fn, device="cuda")
    bt = torch.zeros((1, 1), dtype=torch.int32, device="cuda")
    cl = torch.ones(1, dtype=torch.int32, device="cuda")
    with pytest.raises(ops.CacheFlowError) as e:  # head_dim 64
        ops.paged_attention_fp8_v1(torch.empty_like(q), q, kc, kc, bt, cl, 1.0, 1.0)
    assert e.value.status == _lib.CF_ERR_UNSUPPORTED
    q = torch.zeros((1, 8, 128), dtype=torch.float16, device="cuda")
    kc = torch.zeros((2, 8, 16, 128), dtype=torch.float8_e4m3fn, device="cuda")
    with pytest.raises(ops.CacheFlowError) as e:  # scale must be finite and > 0
        ops.paged_attention_fp8_v1(torch.empty_like(q), q, kc, kc, bt, cl, 0.0, 1.0)
    assert e.value.status == _lib.CF_ERR_INVALID_ARGUMENT
