"""Chunked-prefill attention (cf_paged_prefill_attention) against the oracle:
every query token of a chunk must equal a decode row with context length =
its position + 1 over the same block table."""

import math

import numpy as np
import pytest

from cacheflow_b200.workloads import host_values
from helpers import CODE, as_f64, assert_close, random_tables, to_dev, torch_dtype

pytestmark = pytest.mark.gpu

CONSUMERS = ["mma", "tc"]


@pytest.fixture(params=CONSUMERS)
def consumer(request, monkeypatch):
    """Selects the prefill kernel: mma.sync warps or tcgen05 with tensor memory."""
    monkeypatch.setenv("CF_PREFILL_CONSUMER", request.param)
    return request.param


def _case(rng, dtype, H, Hkv, D, chunks):
    """chunks: list of (tokens already cached, chunk length)."""
    ctx = [pre + n for pre, n in chunks]
    pool = sum((c + 15) // 16 for c in ctx) + 6
    tables = random_tables(rng, ctx, pool)
    qs = np.zeros(len(chunks) + 1, np.int32)
    qs[1:] = np.cumsum([n for _, n in chunks])
    q = host_values((int(qs[-1]), H, D), dtype, 0.5, rng)
    k = host_values((pool, Hkv, 16, D), dtype, 0.5, rng)
    v = host_values((pool, Hkv, 16, D), dtype, 0.5, rng)
    return q, k, v, tables, np.array(ctx, np.int32), qs


def _rows(tables, ctx, qs):
    """The equivalent decode rows: one per query token, causal context length."""
    rt, rc = [], []
    for c in range(len(ctx)):
        n = int(qs[c + 1] - qs[c])
        for i in range(n):
            rt.append(tables[c])
            rc.append(int(ctx[c]) - n + i + 1)
    return np.stack(rt).astype(np.int32), np.array(rc, np.int32)


def _run(ops, dtype, q, k, v, tables, ctx, qs):
    import torch

    dq, dk, dv = to_dev(q, dtype), to_dev(k, dtype), to_dev(v, dtype)
    out = torch.full(dq.shape, 7.0, dtype=torch_dtype(dtype), device="cuda")
    ops.paged_prefill_attention(out, dq, dk, dv, to_dev(tables), to_dev(ctx), to_dev(qs))
    return out, (dq, dk, dv)


CASES = [
    # dtype, H, Hkv, D, chunks (cached tokens, chunk length)
    ("bf16", 32, 8, 128, [(0, 1), (0, 17), (5, 1), (100, 64), (1000, 512), (16, 16), (2047, 300)]),
    ("f16", 32, 8, 128, [(0, 600), (333, 31)]),
    ("bf16", 8, 8, 128, [(0, 100), (4000, 129), (15, 2)]),
    ("bf16", 16, 2, 128, [(7, 70), (1500, 33)]),
    ("f16", 12, 4, 64, [(0, 45), (900, 200)]),  # group of 3: 21 tokens per tile
    ("f16", 8, 8, 128, [(0, 100), (15, 2), (4000, 129)]),  # f16 P without a remainder: short rows too
    ("bf16", 64, 1, 64, [(50, 9), (0, 3)]),     # group of 64: one token per tile
]


@pytest.mark.parametrize("dtype,H,Hkv,D,chunks", CASES)
def test_prefill_matches_oracle_rows(cflib, oracle_mod, consumer, dtype, H, Hkv, D, chunks):
    from cacheflow_b200 import ops

    rng = np.random.default_rng(hash((dtype, H, Hkv, D, len(chunks))) % 2**32)
    q, k, v, tables, ctx, qs = _case(rng, dtype, H, Hkv, D, chunks)
    out, _ = _run(ops, dtype, q, k, v, tables, ctx, qs)
    rt, rc = _rows(tables, ctx, qs)
    want = oracle_mod.paged_attention(q, k, v, rt, rc, 1 / math.sqrt(D), CODE[dtype], num_threads=8)
    assert_close(as_f64(out), want, dtype, "prefill")
    assert ops.device_errors(0) == 0


def test_prefill_agrees_with_decode_rows(cflib, consumer):
    """The decode kernel on the per-token rows gives the same answer (within
    twice the tolerance: each is within it of the truth)."""
    import torch

    from cacheflow_b200 import ops

    rng = np.random.default_rng(5)
    q, k, v, tables, ctx, qs = _case(rng, "bf16", 32, 8, 128, [(600, 300), (0, 40)])
    out, (dq, dk, dv) = _run(ops, "bf16", q, k, v, tables, ctx, qs)
    rt, rc = _rows(tables, ctx, qs)
    rows = torch.empty_like(out)
    ops.paged_attention_v1(rows, dq, dk, dv, to_dev(rt), to_dev(rc), None, int(rc.max()))
    err = (rows.double() - out.double()).abs()
    assert bool((err <= 4e-3 + 2e-3 * out.double().abs()).all()), err.max().item()


def test_prefill_ignores_garbage_past_context(cflib, oracle_mod, consumer):
    import torch

    from cacheflow_b200 import ops

    rng = np.random.default_rng(6)
    q, k, v, tables, ctx, qs = _case(rng, "f16", 16, 4, 128, [(10, 20), (3, 50)])
    dq, dk, dv = to_dev(q, "f16"), to_dev(k, "f16"), to_dev(v, "f16")
    for c in range(len(ctx)):
        if ctx[c] % 16:
            b = tables[c][ctx[c] // 16]
            dk[b, :, ctx[c] % 16:] = float("nan")
            dv[b, :, ctx[c] % 16:] = float("nan")
    out = torch.empty_like(dq)
    ops.paged_prefill_attention(out, dq, dk, dv, to_dev(tables), to_dev(ctx), to_dev(qs))
    rt, rc = _rows(tables, ctx, qs)
    want = oracle_mod.paged_attention(q, k, v, rt, rc, 1 / math.sqrt(128), CODE["f16"])
    assert_close(as_f64(out), want, "f16", "prefill with NaN past the context")


@pytest.mark.parametrize("slope", [1 / 64, 1 / 256, -1 / 64])
def test_prefill_scores_that_grow_along_the_context(cflib, oracle_mod, consumer, slope):
    """Keys whose scores rise (or fall) steadily with position: the running row
    maximum moves by about 16 (or 4) in log2 units per 64-key stage, which
    exercises the deferred rescale of the output accumulator."""
    from cacheflow_b200 import ops

    rng = np.random.default_rng(11)
    H, Hkv, D = 16, 4, 128
    q, k, v, tables, ctx, qs = _case(rng, "f16", H, Hkv, D, [(0, 300), (500, 200), (37, 5)])
    q = (1.0 + 0.05 * rng.standard_normal(q.shape)).astype(np.float16)
    for c in range(len(ctx)):
        pos = np.arange(int(ctx[c]))
        b, o = tables[c][pos // 16], pos % 16
        base = (slope * pos if slope > 0 else slope * (pos - ctx[c]))[:, None, None]
        k[b, :, o, :] = (base + 0.05 * rng.standard_normal((len(pos), Hkv, D))).astype(np.float16)
    out, _ = _run(ops, "f16", q, k, v, tables, ctx, qs)
    rt, rc = _rows(tables, ctx, qs)
    want = oracle_mod.paged_attention(q, k, v, rt, rc, 1 / math.sqrt(D), CODE["f16"], num_threads=8)
    assert_close(as_f64(out), want, "f16", f"prefill, slope {slope}")
    assert ops.device_errors(0) == 0


def test_prefill_bad_block_id_is_recorded(cflib, consumer):
    from cacheflow_b200 import _lib, ops

    rng = np.random.default_rng(8)
    q, k, v, tables, ctx, qs = _case(rng, "bf16", 8, 8, 128, [(40, 10)])
    tables[0, 1] = k.shape[0] + 3
    ops.device_errors(0, clear=True)
    _run(ops, "bf16", q, k, v, tables, ctx, qs)
    assert ops.device_errors(0, clear=True) & _lib.CF_DEVERR_BLOCK_ID


def test_prefill_rejects_fp32_and_bad_shapes(cflib):
    import torch

    from cacheflow_b200 import _lib, ops

    q = torch.zeros((4, 8, 128), device="cuda")
    k = torch.zeros((4, 8, 16, 128), device="cuda")
    bt = torch.zeros((1, 1), dtype=torch.int32, device="cuda")
    cl = torch.tensor([4], dtype=torch.int32, device="cuda")
    qs = torch.tensor([0, 4], dtype=torch.int32, device="cuda")
    with pytest.raises(ops.CacheFlowError) as e:
        ops.paged_prefill_attention(torch.empty_like(q), q, k, k, bt, cl, qs)
    assert e.value.status == _lib.CF_ERR_UNSUPPORTED
