"""The CPU oracle checked on its own: against an independent numpy restatement,
against the golden vectors recorded from CacheFlow's own kernels
(tests/golden/), and for the algebraic identities the path relies on."""

import math
from pathlib import Path

import numpy as np
import pytest

from cacheflow_b200 import workloads
from cacheflow_b200.workloads import host_values
from helpers import CODE, random_tables

GOLDEN = Path(__file__).resolve().parent / "golden"


def _case(rng, dtype, S, H, Hkv, D, ctx):
    pool = sum((c + 15) // 16 for c in ctx) + 5
    tables = random_tables(rng, ctx, pool)
    q = host_values((S, H, D), dtype, 0.5, rng)
    k = host_values((pool, Hkv, 16, D), dtype, 0.5, rng)
    v = host_values((pool, Hkv, 16, D), dtype, 0.5, rng)
    return q, k, v, tables, np.array(ctx, np.int32)


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("H,Hkv,D", [(4, 4, 128), (8, 2, 64), (6, 3, 128)])
def test_c_oracle_matches_numpy_restatement(oracle_mod, dtype, H, Hkv, D):
    rng = np.random.default_rng(1)
    ctx = [1, 15, 16, 17, 100, 300]
    q, k, v, tables, cl = _case(rng, dtype, len(ctx), H, Hkv, D, ctx)
    scale = 1 / math.sqrt(D)
    a = oracle_mod.paged_attention(q, k, v, tables, cl, scale, CODE[dtype])
    b = oracle_mod.paged_attention_numpy(q, k, v, tables, cl, scale, CODE[dtype])
    np.testing.assert_allclose(a, b, rtol=1e-12, atol=1e-12)
    a4 = oracle_mod.paged_attention(q, k, v, tables, cl, scale, CODE[dtype], num_threads=4)
    assert np.array_equal(a, a4)


def test_element_decoding(oracle_mod):
    x = np.array([0.0, -1.5, 65504.0, 6.1e-5, 5.96e-8, np.inf], np.float16)
    for i, val in enumerate(x):
        assert oracle_mod.lib().cfo_load(x.ctypes.data, i, 1) == float(val)
    f = np.array([1.0, -3.140625, 1e-20, 3.0e38], np.float32)
    bits = (f.view(np.uint32) >> 16).astype(np.uint16)  # exact in bf16 for these values? truncate
    for i in range(len(f)):
        want = float((bits[i:i + 1].astype(np.uint32) << 16).view(np.float32)[0])
        assert oracle_mod.lib().cfo_load(bits.ctypes.data, i, 2) == want


def test_bf16_rounding_is_round_to_nearest_even():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5e-3], np.float32)  # ties and a normal value
    bits = host_values_rounding(x)
    import torch

    want = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(bits, want)


def host_values_rounding(x):
    u = x.view(np.uint32)
    r = ((u >> 16) & 1) + np.uint32(0x7FFF)
    return ((u + r) >> 16).astype(np.uint16)


@pytest.mark.parametrize("P", [16, 64, 512])
def test_partitions_then_reduce_equals_direct(oracle_mod, P):
    rng = np.random.default_rng(2)
    ctx = [1, P - 1, P, P + 1, 5 * P + 3]
    q, k, v, tables, cl = _case(rng, "bf16", len(ctx), 8, 2, 128, ctx)
    scale = 1 / math.sqrt(128)
    nparts = (max(ctx) + P - 1) // P
    mx, es, to = oracle_mod.paged_attention_partitions(q, k, v, tables, cl, scale, P, nparts, 2)
    red = oracle_mod.paged_attention_reduce(mx, es, to, cl, P)
    direct = oracle_mod.paged_attention(q, k, v, tables, cl, scale, 2)
    np.testing.assert_allclose(red, direct, rtol=1e-12, atol=1e-13)


def test_zero_context_is_zero(oracle_mod):
    rng = np.random.default_rng(3)
    q, k, v, tables, cl = _case(rng, "f32", 2, 2, 2, 64, [0, 5])
    out = oracle_mod.paged_attention(q, k, v, tables, cl, 0.125, 0)
    assert np.all(out[0] == 0) and np.all(np.isfinite(out[1]))


def test_cache_ops_match_numpy(oracle_mod):
    rng = np.random.default_rng(4)
    pool, Hkv, D, T = 30, 4, 64, 40
    kc = host_values((pool, Hkv, 16, D), "bf16", 1.0, rng)
    vc = host_values((pool, Hkv, 16, D), "bf16", 1.0, rng)
    key = host_values((T, Hkv, D), "bf16", 1.0, rng)
    val = host_values((T, Hkv, D), "bf16", 1.0, rng)
    slots = rng.permutation(pool * 16)[:T].astype(np.int32)
    slots[3] = -1
    ek, ev = kc.copy(), vc.copy()
    ok = slots >= 0
    ek[slots[ok] // 16, :, slots[ok] % 16] = key[ok]
    ev[slots[ok] // 16, :, slots[ok] % 16] = val[ok]
    oracle_mod.reshape_and_cache(key, val, kc, vc, slots)
    assert np.array_equal(kc, ek) and np.array_equal(vc, ev)

    ids = rng.permutation(pool)
    pairs = np.stack([ids[:6], ids[6:12]], 1)
    ek[pairs[:, 1]] = ek[pairs[:, 0]]
    ev[pairs[:, 1]] = ev[pairs[:, 0]]
    oracle_mod.copy_blocks(kc, vc, pairs)
    assert np.array_equal(kc, ek) and np.array_equal(vc, ev)

    other = np.zeros_like(kc)
    oracle_mod.swap_blocks(kc, other, pairs)
    want = np.zeros_like(kc)
    want[pairs[:, 1]] = kc[pairs[:, 0]]
    assert np.array_equal(other, want)

    src, dst = np.array([20, 21, 5], np.int32), np.array([2, 3, 5], np.int32)
    ek[dst], ev[dst] = ek[src], ev[src]
    oracle_mod.compact_kv_cache(kc, vc, src, dst)
    assert np.array_equal(kc, ek) and np.array_equal(vc, ev)

    oracle_mod.memset_blocks(kc, np.array([0, 29], np.int32))
    ek[[0, 29]] = 0
    assert np.array_equal(kc, ek)


def test_compact_oracle_is_parallel_assignment(oracle_mod):
    """A swap cycle (which races in the concurrent reference kernel) is defined
    as: every destination receives its source's contents from before the call."""
    c = np.arange(4 * 16 * 2, dtype=np.float32).reshape(4, 1, 16, 2)
    v = c.copy()
    before = c.copy()
    oracle_mod.compact_kv_cache(c, v, np.array([0, 1], np.int32), np.array([1, 0], np.int32))
    assert np.array_equal(c[0], before[1]) and np.array_equal(c[1], before[0])


@pytest.mark.parametrize("name", list(workloads.WORKLOADS))
def test_workload_generators_are_consistent(name):
    w = workloads.make(name)
    w2 = workloads.make(name)
    assert np.array_equal(w.context_lens, w2.context_lens) and np.array_equal(w.block_tables, w2.block_tables)
    nblk = (w.context_lens.astype(np.int64) + 15) // 16
    assert nblk.max() <= w.block_tables.shape[1]
    for s in range(w.num_seqs):
        row = w.block_tables[s, : nblk[s]]
        assert row.min() >= 0 and row.max() < w.num_blocks
    # every new token has its own slot, inside the pool, inside its row's blocks
    assert len(np.unique(w.slot_mapping)) == len(w.slot_mapping)
    assert w.slot_mapping.min() >= 0 and w.slot_mapping.max() < w.num_blocks * 16
    for slot, r in zip(w.slot_mapping[:50], w.slot_rows[:50]):
        pos = w.context_lens[r] - 1
        assert slot == w.block_tables[r, pos // 16] * 16 + pos % 16


def test_workload_sizes_match_the_configs():
    assert workloads.make("cpu_decode_fp32").num_blocks == 512
    w = workloads.make("llama2_7b_ragged_decode")
    assert w.num_seqs == 64 and 1.9e9 < w.kv_bytes() < 2.5e9
    w = workloads.make("llama3_8b_long_decode")
    assert w.num_seqs == 16 and w.context_lens.min() >= 16384 and w.context_lens.max() <= 131072
    w = workloads.make("continuous_batching_mixed")
    assert w.num_seqs == 224 + 32 * 512 and len(w.slot_mapping) == 16608 and len(w.copy_pairs) == 16
    assert w.unique_kv_bytes() < w.kv_bytes()


GOLDEN_FILES = sorted(GOLDEN.glob("*.npz"))


@pytest.mark.skipif(not GOLDEN_FILES, reason="no golden vectors recorded")
@pytest.mark.parametrize("path", GOLDEN_FILES, ids=lambda p: p.stem)
def test_oracle_reproduces_golden_vectors(oracle_mod, path):
    """Golden outputs were produced by CacheFlow's own CUDA kernels
    (tests/golden/make_golden.py) and its own host code
    (tests/golden/make_golden_cpu.py); the oracle must reproduce them."""
    g = dict(np.load(path))
    op = str(g["op"])
    if op == "paged_attention_v1":
        out = oracle_mod.paged_attention(g["q"], g["k"], g["v"], g["block_tables"], g["context_lens"],
                                         float(g["scale"]), 0)
        np.testing.assert_allclose(out, g["out"], rtol=1e-5, atol=1e-5)
    elif op == "reshape_and_cache":
        kc, vc = g["k_cache"].copy(), g["v_cache"].copy()
        oracle_mod.reshape_and_cache(g["key"], g["value"], kc, vc, g["slot_mapping"])
        assert np.array_equal(kc, g["k_out"]) and np.array_equal(vc, g["v_out"])
    elif op == "copy_blocks":
        kc, vc = g["k_cache"].copy(), g["v_cache"].copy()
        oracle_mod.copy_blocks(kc, vc, g["block_mapping"])
        assert np.array_equal(kc, g["k_out"]) and np.array_equal(vc, g["v_out"])
    elif op == "swap_blocks":
        dst = g["dst"].copy()
        oracle_mod.swap_blocks(g["src"], dst, g["block_mapping"])
        assert np.array_equal(dst, g["dst_out"])
    elif op == "compact_kv_cache":
        kc, vc = g["k_cache"].copy(), g["v_cache"].copy()
        oracle_mod.compact_kv_cache(kc, vc, g["src_ids"], g["dst_ids"])
        assert np.array_equal(kc, g["k_out"]) and np.array_equal(vc, g["v_out"])
    elif op == "build_decode_inputs":
        tables, ctx, slots, cut = oracle_mod.build_decode_inputs(
            g["positions"], g["block_offsets"], g["block_ids"], g["block_tables"].shape[1])
        assert cut == 0
        assert np.array_equal(tables, g["block_tables"]) and np.array_equal(ctx, g["context_lens"])
        assert np.array_equal(slots, g["slot_mapping"])
        assert np.all(slots[~g["slot_set"]] == -1)
    elif op == "memset_blocks":
        c = g["cache"].copy()
        oracle_mod.memset_blocks(c, g["block_ids"])
        assert np.array_equal(c, g["out"])
    else:
        pytest.fail(f"unknown golden op {op}")


def test_build_decode_inputs_edge_cases(oracle_mod):
    """Negative positions are empty rows; rows longer than the table width are
    cut (and counted); a position past the row's blocks gets slot -1."""
    pos = np.array([-1, 0, 40, 5, 100], np.int32)
    nblk = np.array([2, 1, 3, 6, 2], np.int64)
    off = np.concatenate([[0], np.cumsum(nblk)]).astype(np.int64)
    ids = np.arange(100, 100 + int(off[-1]), dtype=np.int32)
    tables, ctx, slots, cut = oracle_mod.build_decode_inputs(pos, off, ids, 4)
    assert cut == 1
    assert ctx.tolist() == [0, 1, 41, 6, 101]
    assert slots.tolist() == [-1, 102 * 16, 105 * 16 + 8, 106 * 16 + 5, -1]
    assert tables[3].tolist() == [106, 107, 108, 109] and tables[1].tolist() == [102, 0, 0, 0]


def test_e4m3_codec_matches_torch(oracle_mod):
    """The oracle's e4m3 decoding of all 256 codes and its rounding (nearest,
    ties to even) agree with torch.float8_e4m3fn, an independent
    implementation of the OCP format; saturation is the oracle's own rule."""
    import torch

    codes = np.arange(256, dtype=np.uint8)
    ours = oracle_mod.e4m3_to_float(codes)
    theirs = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy().astype(np.float64)
    assert np.array_equal(np.isnan(ours), np.isnan(theirs))
    ok = ~np.isnan(ours)
    assert np.array_equal(ours[ok], theirs[ok])
    # values: random magnitudes over the whole range, exact codes, midpoints
    # between neighbouring codes (ties), subnormals, signed zeros
    rng = np.random.default_rng(8)
    finite = np.sort(np.unique(np.abs(ours[ok])))
    mids = (finite[:-1] + finite[1:]) / 2
    x = np.concatenate([
        rng.uniform(-447.9, 447.9, 3000), rng.standard_normal(3000) * 0.01, finite, -finite, mids, -mids,
        rng.uniform(0, 2 ** -6, 500), [0.0, -0.0],
    ]).astype(np.float32)
    x = x[np.abs(x) < 448]
    got = oracle_mod.e4m3_from_float(x)
    want = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(got, want)
    # saturation (the kernels' satfinite conversion): +-448 and beyond, infinities
    big = np.array([448.0, 449.0, 464.0, 500.0, 1e30, np.inf], np.float32)
    assert np.all(oracle_mod.e4m3_from_float(big) == 0x7E)
    assert np.all(oracle_mod.e4m3_from_float(-big) == 0xFE)


@pytest.mark.parametrize("qdtype", ["f16", "bf16"])
def test_fp8_attention_oracle_equals_dequantized_attention(oracle_mod, qdtype):
    rng = np.random.default_rng(9)
    ctx = [1, 16, 17, 300]
    S, H, Hkv, D = len(ctx), 8, 2, 128
    pool = sum((c + 15) // 16 for c in ctx) + 3
    tables = random_tables(rng, ctx, pool)
    q = host_values((S, H, D), qdtype, 0.5, rng)
    codes = rng.integers(0, 256, (2, pool, Hkv, 16, D)).astype(np.uint8)
    codes[(codes & 0x7F) == 0x7F] = 0x3C  # no NaN codes
    kc, vc = codes[0], codes[1]
    ks, vs = 0.02, 0.05
    got = oracle_mod.paged_attention_fp8(q, kc, vc, tables, np.array(ctx, np.int32), 1 / math.sqrt(D), ks, vs,
                                         CODE[qdtype])
    # the scales reach the oracle as float32
    kd = oracle_mod.e4m3_to_float(kc) * float(np.float32(ks))
    vd = oracle_mod.e4m3_to_float(vc) * float(np.float32(vs))
    qd = oracle_mod.to_f64(q, CODE[qdtype])
    want = oracle_mod.paged_attention_numpy(qd, kd, vd, tables, np.array(ctx, np.int32), 1 / math.sqrt(D))
    np.testing.assert_allclose(got, want, rtol=1e-12, atol=1e-12)


def test_fp8_reshape_oracle(oracle_mod):
    rng = np.random.default_rng(10)
    T, Hkv, D, pool = 6, 2, 32, 4
    key = host_values((T, Hkv, D), "bf16", 3.0, rng)
    val = host_values((T, Hkv, D), "bf16", 3.0, rng)
    kc = np.zeros((pool, Hkv, 16, D), np.uint8)
    vc = np.zeros_like(kc)
    slots = np.array([0, 17, 33, -1, 63, 5], np.int32)
    oracle_mod.reshape_and_cache_fp8(key, val, kc, vc, slots, 0.5, 0.25, CODE["bf16"])
    kf = oracle_mod.to_f64(key, CODE["bf16"]).astype(np.float32)
    for t, s in enumerate(slots):
        if s < 0:
            continue
        want = oracle_mod.e4m3_from_float(kf[t] / np.float32(0.5))
        assert np.array_equal(kc[s // 16, :, s % 16], want)
    assert not kc[0, :, 1:5].any()
