"""Fused append + attention (cf_paged_attention_append_v1/_v2) against the
unfused pair it replaces -- cf_reshape_and_cache of every row's newest token,
then cf_paged_attention_v1/_v2 -- and against the oracle; and the device-side
decode-input builder (cf_build_decode_inputs) against the oracle's
restatement of prepare_kv_cache_inputs."""

import math

import numpy as np
import pytest

from cacheflow_b200.workloads import host_values
from helpers import CODE, as_f64, assert_close, random_tables, to_dev, torch_dtype

pytestmark = pytest.mark.gpu

CASES = [
    # dtype, num_heads, num_kv_heads, head_dim, context lengths (new token included)
    ("f32", 4, 4, 128, [1, 15, 16, 17, 129, 600]),
    ("f32", 8, 2, 64, [1, 33, 1700]),
    ("f16", 8, 8, 128, [1, 16, 17, 512, 513, 2049]),
    ("bf16", 32, 8, 128, [1, 2, 16, 17, 1025, 4000]),   # group 4: tensor-core consumer
    ("bf16", 32, 2, 128, [3, 160, 1030]),               # group 16: two head chunks per kv head
    ("f16", 12, 4, 64, [1, 100, 1500]),
    ("bf16", 8, 8, 256, [1, 17, 300]),
]


def _setup(rng, dtype, H, Hkv, D, ctx):
    S = len(ctx)
    pool = sum((c + 15) // 16 for c in ctx) + 5
    tables = random_tables(rng, ctx, pool)
    q = host_values((S, H, D), dtype, 0.5, rng)
    k = host_values((pool, Hkv, 16, D), dtype, 0.5, rng)
    v = host_values((pool, Hkv, 16, D), dtype, 0.5, rng)
    nk = host_values((S, Hkv, D), dtype, 0.5, rng)
    nv = host_values((S, Hkv, D), dtype, 0.5, rng)
    ctx = np.array(ctx, np.int32)
    pos = ctx - 1
    slots = (tables[np.arange(S), pos // 16] * 16 + pos % 16).astype(np.int32)
    return q, k, v, nk, nv, tables, ctx, slots


def _dev(dtype, *arrays):
    return [to_dev(a, dtype) for a in arrays]


@pytest.fixture(params=["auto", "fma", "mma"])
def consumer(request, monkeypatch):
    if request.param == "auto":
        monkeypatch.delenv("CF_ATTN_CONSUMER", raising=False)
    else:
        monkeypatch.setenv("CF_ATTN_CONSUMER", request.param)
    return request.param


@pytest.mark.parametrize("path", ["v1", "v1_split", "v2"])
@pytest.mark.parametrize("dtype,H,Hkv,D,ctx", CASES)
def test_append_equals_reshape_then_attention(cflib, oracle_mod, consumer, path, dtype, H, Hkv, D, ctx):
    import torch

    from cacheflow_b200 import ops

    if consumer != "auto" and dtype == "f32":
        pytest.skip("fp32 caches always use the FMA consumer")
    rng = np.random.default_rng(hash((dtype, H, Hkv, D, len(ctx), path)) % 2**32)
    q, k, v, nk, nv, tables, cl, slots = _setup(rng, dtype, H, Hkv, D, ctx)
    dq, dnk, dnv = _dev(dtype, q, nk, nv)
    bt, dcl, dsl = to_dev(tables), to_dev(cl), to_dev(slots)
    mctx = int(cl.max())
    S = len(ctx)

    def run(fused, with_slots):
        dk, dv = _dev(dtype, k, v)
        out = torch.full((S, H, D), 3.0, dtype=torch_dtype(dtype), device="cuda")
        sl = dsl if with_slots else None
        if path == "v2":
            P = ops.v2_num_partitions(mctx)
            es = torch.empty((S, H, P), device="cuda")
            ml = torch.empty_like(es)
            to = torch.empty((S, H, P, D), device="cuda")
            if fused:
                ops.paged_attention_append_v2(out, es, ml, to, dq, dnk, dnv, dk, dv, bt, dcl, sl)
            else:
                ops.reshape_and_cache(dnk, dnv, dk, dv, dsl)
                ops.paged_attention_v2(out, es, ml, to, dq, dk, dv, bt, dcl)
        else:
            ws = None
            if path == "v1_split":
                n = ops.paged_attention_v1_workspace_size(dq, dk, bt, mctx)
                ws = torch.empty(max(n, 16), dtype=torch.uint8, device="cuda") if n else None
            if fused:
                ops.paged_attention_append_v1(out, dq, dnk, dnv, dk, dv, bt, dcl, sl, workspace=ws)
            else:
                ops.reshape_and_cache(dnk, dnv, dk, dv, dsl)
                ops.paged_attention_v1(out, dq, dk, dv, bt, dcl, workspace=ws)
        return out, dk, dv

    ops.device_errors(0, clear=True)
    o_ref, k_ref, v_ref = run(False, True)
    for with_slots in (False, True):
        o, kk, vv = run(True, with_slots)
        assert torch.equal(kk, k_ref) and torch.equal(vv, v_ref), "cache after the fused append"
        assert torch.equal(o, o_ref), "fused output differs from reshape + attention"
    assert ops.device_errors(0) == 0
    # and the oracle on the appended cache
    k2, v2 = k.copy(), v.copy()
    oracle_mod.reshape_and_cache(nk, nv, k2, v2, slots)
    want = oracle_mod.paged_attention(q, k2, v2, tables, cl, 1 / math.sqrt(D), CODE[dtype], num_threads=4)
    assert_close(as_f64(o_ref), want, dtype, f"append {path}")


def test_negative_and_wrong_slots_append_nothing(cflib, oracle_mod):
    import torch

    from cacheflow_b200 import _lib, ops

    rng = np.random.default_rng(3)
    q, k, v, nk, nv, tables, cl, slots = _setup(rng, "bf16", 32, 8, 128, [20, 33, 700, 64])
    bad = slots.copy()
    bad[1] = -7                      # any negative slot: the row appends nothing
    bad[2] = slots[2] + 1            # not the slot of its newest position
    dq, dk, dv, dnk, dnv = _dev("bf16", q, k, v, nk, nv)
    out = torch.empty((4, 32, 128), dtype=torch.bfloat16, device="cuda")
    ops.device_errors(0, clear=True)
    ops.paged_attention_append_v1(out, dq, dnk, dnv, dk, dv, to_dev(tables), to_dev(cl), to_dev(bad))
    assert ops.device_errors(0, clear=True) == _lib.CF_DEVERR_SLOT
    k2, v2 = k.copy(), v.copy()
    ok = np.array([True, False, False, True])
    oracle_mod.reshape_and_cache(nk[ok], nv[ok], k2, v2, slots[ok])
    from helpers import to_host

    assert np.array_equal(to_host(dk), k2) and np.array_equal(to_host(dv), v2)
    want = oracle_mod.paged_attention(q, k2, v2, tables, cl, 1 / math.sqrt(128), CODE["bf16"], num_threads=4)
    assert_close(as_f64(out), want, "bf16", "rows that append nothing attend to the cache as it is")


def test_append_rejects_misaligned_and_missing_rows(cflib):
    import torch

    from cacheflow_b200 import _lib, ops

    q = torch.zeros((2, 4, 128), dtype=torch.float16, device="cuda")
    kc = torch.zeros((4, 4, 16, 128), dtype=torch.float16, device="cuda")
    bt = torch.zeros((2, 1), dtype=torch.int32, device="cuda")
    cl = torch.ones(2, dtype=torch.int32, device="cuda")
    nk = torch.zeros((2, 4, 128), dtype=torch.float16, device="cuda")
    p = ops._attention_params(torch.empty_like(q), q, kc, kc, bt, cl, 0.1, 1)
    lib = _lib.load()
    import ctypes

    assert lib.cf_paged_attention_append_v1(ctypes.byref(p), None, nk.data_ptr(), None, None, 0, None) == \
        _lib.CF_ERR_INVALID_ARGUMENT
    assert lib.cf_paged_attention_append_v1(ctypes.byref(p), nk.data_ptr() + 2, nk.data_ptr(), None, None, 0,
                                            None) == _lib.CF_ERR_INVALID_ARGUMENT
    with pytest.raises(ops.CacheFlowError):
        ops.paged_attention_append_v1(torch.empty_like(q), q, nk[:1], nk[:1], kc, kc, bt, cl)


def _csr(rng, S, max_blocks):
    nblk = rng.integers(0, max_blocks + 1, S)
    pos = np.array([int(rng.integers(-1, max(n, 1) * 16 + 8)) for n in nblk], np.int32)
    off = np.zeros(S + 1, np.int64)
    off[1:] = np.cumsum(nblk)
    ids = rng.permutation(10_000_000)[: int(off[-1])].astype(np.int32)
    return pos, off, ids


@pytest.mark.parametrize("S,max_blocks", [(1, 1), (7, 3), (300, 40), (64, 2048), (1024, 300)])
def test_build_decode_inputs_matches_oracle(cflib, oracle_mod, S, max_blocks):
    from cacheflow_b200 import ops
    from helpers import to_host

    rng = np.random.default_rng(S * 7919 + max_blocks)
    pos, off, ids = _csr(rng, S, max_blocks)
    ops.device_errors(0, clear=True)
    bt, cl, sl = ops.build_decode_inputs(to_dev(pos), to_dev(off), to_dev(ids), max_blocks)
    t, c, s, cut = oracle_mod.build_decode_inputs(pos, off, ids, max_blocks)
    assert cut == 0 and ops.device_errors(0) == 0
    assert np.array_equal(to_host(bt), t) and np.array_equal(to_host(cl), c) and np.array_equal(to_host(sl), s)


def test_build_decode_inputs_golden_and_cut_rows(cflib, oracle_mod):
    from pathlib import Path

    from cacheflow_b200 import _lib, ops
    from helpers import to_host

    g = dict(np.load(Path(__file__).resolve().parent / "golden" / "build_decode_inputs.npz"))
    mb = g["block_tables"].shape[1]
    bt, cl, sl = ops.build_decode_inputs(to_dev(g["positions"]), to_dev(g["block_offsets"]),
                                         to_dev(g["block_ids"]), mb)
    assert np.array_equal(to_host(bt), g["block_tables"]) and np.array_equal(to_host(cl), g["context_lens"])
    assert np.array_equal(to_host(sl), g["slot_mapping"])
    # narrower tables than the widest row: rows are cut and the cut is recorded
    ops.device_errors(0, clear=True)
    bt, cl, sl = ops.build_decode_inputs(to_dev(g["positions"]), to_dev(g["block_offsets"]),
                                         to_dev(g["block_ids"]), 8)
    t, c, s, cut = oracle_mod.build_decode_inputs(g["positions"], g["block_offsets"], g["block_ids"], 8)
    assert cut > 0 and ops.device_errors(0, clear=True) == _lib.CF_DEVERR_CONTEXT_LEN
    assert np.array_equal(to_host(bt), t) and np.array_equal(to_host(cl), c) and np.array_equal(to_host(sl), s)
