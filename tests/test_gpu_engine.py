"""The host-side decode step (cacheflow_b200.engine.DecodeEngine.step) from
pinned host buffers: pipelined steps give the oracle's answer, and the fused
append path equals reshape_and_cache + attention bit for bit."""

import math

import numpy as np
import pytest

from cacheflow_b200.workloads import host_values
from helpers import CODE, as_f64, assert_close, random_tables, to_dev, to_host

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kernel", ["v1", "reference"])
@pytest.mark.parametrize("dtype,H,Hkv,D,ctx", [
    ("f16", 8, 8, 128, [1, 17, 300, 2000]),
    ("bf16", 32, 8, 128, [5, 16, 9000, 700]),   # longest > 8192: v1 split at 2048, or v2 ("reference")
])
def test_engine_steps_fused_and_separate(cflib, oracle_mod, dtype, H, Hkv, D, ctx, kernel):
    import torch

    from cacheflow_b200.engine import DecodeEngine

    rng = np.random.default_rng(17)
    S = len(ctx)
    steps = 3
    pool = sum((c + steps + 15) // 16 for c in ctx) + 4
    tables = random_tables(rng, [c + steps for c in ctx], pool)
    k0 = host_values((pool, Hkv, 16, D), dtype, 0.5, rng)
    v0 = host_values((pool, Hkv, 16, D), dtype, 0.5, rng)
    qs = [host_values((S, H, D), dtype, 0.5, rng) for _ in range(steps)]
    nks = [host_values((S, Hkv, D), dtype, 0.5, rng) for _ in range(steps)]
    nvs = [host_values((S, Hkv, D), dtype, 0.5, rng) for _ in range(steps)]
    results = {}
    for fused in (False, True):
        dk, dv = to_dev(k0, dtype), to_dev(v0, dtype)
        eng = DecodeEngine(dk, dv, H, S, tables.shape[1], S, fused_append=fused, depth=2, kernel=kernel)
        assert eng._use_v2(max(ctx) + steps) == (kernel == "reference" and max(ctx) > 8192)
        outs = []
        pins = []
        for i in range(steps):
            cl = np.array(ctx, np.int32) + i + 1  # the new token is counted
            pos = cl - 1
            slots = (tables[np.arange(S), pos // 16] * 16 + pos % 16).astype(np.int32)
            pin = [torch.from_numpy(a).pin_memory() for a in (qs[i], nks[i], nvs[i], slots, tables, cl)]
            if dtype == "bf16":
                pin[:3] = [t.view(torch.bfloat16) for t in pin[:3]]
            o = torch.empty(pin[0].shape, dtype=pin[0].dtype).pin_memory()
            eng.step(*pin, o, int(cl.max()))
            pins.append(pin)
            outs.append(o)
        eng.synchronize()
        results[fused] = ([o.clone() for o in outs], to_host(dk), to_host(dv))
    (o_sep, k_sep, v_sep), (o_fus, k_fus, v_fus) = results[False], results[True]
    assert np.array_equal(k_sep, k_fus) and np.array_equal(v_sep, v_fus)
    for a, b in zip(o_sep, o_fus):
        assert torch.equal(a, b)
    # the oracle, step by step
    k, v = k0.copy(), v0.copy()
    for i in range(steps):
        cl = np.array(ctx, np.int32) + i + 1
        pos = cl - 1
        slots = (tables[np.arange(S), pos // 16] * 16 + pos % 16).astype(np.int32)
        oracle_mod.reshape_and_cache(nks[i], nvs[i], k, v, slots)
        want = oracle_mod.paged_attention(qs[i], k, v, tables, cl, 1 / math.sqrt(D), CODE[dtype], num_threads=4)
        assert_close(as_f64(o_fus[i]), want, dtype, f"engine step {i}")
    assert np.array_equal(k, k_fus) and np.array_equal(v, v_fus)


@pytest.mark.parametrize("dtype,H,Hkv,D,ctx", [
    ("f16", 8, 8, 128, [1, 17, 300, 2000]),
    ("bf16", 32, 8, 128, [5, 16, 9000, 700]),
])
@pytest.mark.parametrize("fused", [False, True])
def test_engine_steps_fp8_caches(cflib, oracle_mod, dtype, H, Hkv, D, ctx, fused):
    import torch

    from cacheflow_b200.engine import DecodeEngine

    rng = np.random.default_rng(19)
    S, steps, ks, vs = len(ctx), 3, 0.01, 0.02
    pool = sum((c + steps + 15) // 16 for c in ctx) + 4
    tables = random_tables(rng, [c + steps for c in ctx], pool)
    x = torch.from_numpy(rng.standard_normal((2, pool, Hkv, 16, D)).astype(np.float32) * 50)
    codes = x.to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    k, v = codes[0].copy(), codes[1].copy()
    dk = torch.from_numpy(k.copy()).cuda().view(torch.float8_e4m3fn)
    dv = torch.from_numpy(v.copy()).cuda().view(torch.float8_e4m3fn)
    tdt = torch.float16 if dtype == "f16" else torch.bfloat16
    eng = DecodeEngine(dk, dv, H, S, tables.shape[1], S, kv_scales=(ks, vs), query_dtype=tdt, fused_append=fused)
    outs = []
    steps_in = []
    for i in range(steps):
        cl = np.array(ctx, np.int32) + i + 1
        pos = cl - 1
        slots = (tables[np.arange(S), pos // 16] * 16 + pos % 16).astype(np.int32)
        q = host_values((S, H, D), dtype, 0.5, rng)
        nk = host_values((S, Hkv, D), dtype, 0.5, rng)
        nv = host_values((S, Hkv, D), dtype, 0.5, rng)
        pin = [torch.from_numpy(a).pin_memory() for a in (q, nk, nv, slots, tables, cl)]
        if dtype == "bf16":
            pin[:3] = [t.view(torch.bfloat16) for t in pin[:3]]
        o = torch.empty(pin[0].shape, dtype=tdt).pin_memory()
        eng.step(*pin, o, int(cl.max()))
        outs.append(o)
        steps_in.append((q, nk, nv, slots, cl))
    eng.synchronize()
    for i, (q, nk, nv, slots, cl) in enumerate(steps_in):
        oracle_mod.reshape_and_cache_fp8(nk, nv, k, v, slots, ks, vs, CODE[dtype])
        want = oracle_mod.paged_attention_fp8(q, k, v, tables, cl, 1 / math.sqrt(D), ks, vs, CODE[dtype],
                                              num_threads=4)
        assert_close(as_f64(outs[i]), want, dtype, f"fp8 engine step {i}")
    assert np.array_equal(dk.view(torch.uint8).cpu().numpy(), k)
