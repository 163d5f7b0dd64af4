"""Parity of the paged decode-attention kernels (v1 unsplit, v1 split, v2 + reduce)
with the CPU oracle, through the C ABI, plus known-answer cases and the
device-side range checks."""

import math

import numpy as np
import pytest

from cacheflow_b200.workloads import host_values
from helpers import CODE, TOL, as_f64, assert_close, random_tables, to_dev, torch_dtype

pytestmark = pytest.mark.gpu

EDGE_CTX = [1, 15, 16, 17, 128, 129, 512, 513]

CASES = [
    # dtype, num_heads, num_kv_heads, head_dim, context lengths
    ("f32", 4, 4, 128, EDGE_CTX),
    ("f32", 8, 2, 64, [1, 33, 200, 1700]),
    ("f32", 8, 1, 128, [5, 300]),
    ("f16", 4, 4, 128, EDGE_CTX + [8192, 8193]),
    ("f16", 6, 2, 64, [1, 17, 100, 1500]),
    ("bf16", 8, 2, 128, EDGE_CTX + [2049, 8193]),
    ("bf16", 16, 2, 128, [1, 16, 31, 700, 1025]),
    ("bf16", 8, 8, 256, [1, 17, 300, 1100]),
    ("f16", 32, 2, 128, [3, 160, 1030]),  # group of 16 query heads per kv head
]


def _setup(rng, dtype, H, Hkv, D, ctx, pool_extra=7):
    import torch

    S = len(ctx)
    pool = sum((c + 15) // 16 for c in ctx) + pool_extra
    tables = random_tables(rng, ctx, pool)
    q = host_values((S, H, D), dtype, 0.5, rng)
    k = host_values((pool, Hkv, 16, D), dtype, 0.5, rng)
    v = host_values((pool, Hkv, 16, D), dtype, 0.5, rng)
    dev = dict(q=to_dev(q, dtype), k=to_dev(k, dtype), v=to_dev(v, dtype),
               bt=to_dev(tables), cl=to_dev(np.array(ctx, np.int32)),
               out=torch.empty((S, H, D), dtype=torch_dtype(dtype), device="cuda"))
    return (q, k, v, tables, np.array(ctx, np.int32)), dev


def _oracle(oracle_mod, host, dtype, scale):
    q, k, v, tables, ctx = host
    return oracle_mod.paged_attention(q, k, v, tables, ctx, scale, dtype_code=CODE[dtype], num_threads=4)


CONSUMERS = ["auto", "fma", "mma"]


def _consumer(monkeypatch, dtype, consumer):
    """Selects the attention consumer (FMA or tensor-core MMA) for 16-bit caches."""
    if consumer != "auto" and dtype == "f32":
        pytest.skip("fp32 caches always use the FMA consumer")
    if consumer == "auto":
        monkeypatch.delenv("CF_ATTN_CONSUMER", raising=False)
    else:
        monkeypatch.setenv("CF_ATTN_CONSUMER", consumer)


@pytest.mark.parametrize("consumer", CONSUMERS)
@pytest.mark.parametrize("dtype,H,Hkv,D,ctx", CASES)
def test_v1_unsplit_matches_oracle(cflib, oracle_mod, monkeypatch, dtype, H, Hkv, D, ctx, consumer):
    from cacheflow_b200 import ops

    _consumer(monkeypatch, dtype, consumer)

    rng = np.random.default_rng(hash((dtype, H, Hkv, D, len(ctx))) % 2**32)
    host, d = _setup(rng, dtype, H, Hkv, D, ctx)
    scale = 1.0 / math.sqrt(D)
    ops.paged_attention_v1(d["out"], d["q"], d["k"], d["v"], d["bt"], d["cl"], scale, max(ctx))
    assert_close(as_f64(d["out"]), _oracle(oracle_mod, host, dtype, scale), dtype, "v1")
    assert ops.device_errors(0) == 0


@pytest.mark.parametrize("consumer", CONSUMERS)
@pytest.mark.parametrize("dtype,H,Hkv,D,ctx", CASES)
def test_v1_split_matches_oracle(cflib, oracle_mod, monkeypatch, dtype, H, Hkv, D, ctx, consumer):
    import torch

    from cacheflow_b200 import ops

    _consumer(monkeypatch, dtype, consumer)

    rng = np.random.default_rng(hash((dtype, H, D, "split")) % 2**32)
    host, d = _setup(rng, dtype, H, Hkv, D, ctx)
    scale = 1.0 / math.sqrt(D)
    n = ops.paged_attention_v1_workspace_size(d["q"], d["k"], d["bt"], max(ctx))
    # these small batches split at 512 or 1024 tokens (the policy halves its
    # 2048-token partitions to fill the GPU): longer contexts always split
    if max(ctx) > 1024:
        assert n > 0
    if max(ctx) <= 512:
        assert n == 0
    ws = torch.empty(max(n, 16), dtype=torch.uint8, device="cuda") if n else None
    ops.paged_attention_v1(d["out"], d["q"], d["k"], d["v"], d["bt"], d["cl"], scale, max(ctx), workspace=ws)
    assert_close(as_f64(d["out"]), _oracle(oracle_mod, host, dtype, scale), dtype, "v1 split")
    assert ops.device_errors(0) == 0


@pytest.mark.parametrize("consumer", CONSUMERS)
@pytest.mark.parametrize("dtype,H,Hkv,D,ctx", CASES)
def test_v2_matches_oracle(cflib, oracle_mod, monkeypatch, dtype, H, Hkv, D, ctx, consumer):
    import torch

    from cacheflow_b200 import ops

    _consumer(monkeypatch, dtype, consumer)

    rng = np.random.default_rng(hash((dtype, H, D, "v2")) % 2**32)
    host, d = _setup(rng, dtype, H, Hkv, D, ctx)
    scale = 1.0 / math.sqrt(D)
    S = len(ctx)
    P = ops.v2_num_partitions(max(ctx)) + 1  # a larger stride than needed is allowed
    es = torch.full((S, H, P), float("nan"), device="cuda")
    ml = torch.full((S, H, P), float("nan"), device="cuda")
    to = torch.full((S, H, P, D), float("nan"), device="cuda")
    ops.paged_attention_v2(d["out"], es, ml, to, d["q"], d["k"], d["v"], d["bt"], d["cl"], scale, max(ctx))
    assert_close(as_f64(d["out"]), _oracle(oracle_mod, host, dtype, scale), dtype, "v2")
    # Partition statistics of multi-partition sequences match the oracle's.
    q, k, v, tables, cl = host
    mx, sm, tmp = oracle_mod.paged_attention_partitions(q, k, v, tables, cl, scale, 512, P, CODE[dtype])
    for s, c in enumerate(ctx):
        parts = (c + 511) // 512
        if parts < 2:
            continue
        np.testing.assert_allclose(ml[s, :, :parts].double().cpu().numpy(), mx[s, :, :parts], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(es[s, :, :parts].double().cpu().numpy(), sm[s, :, :parts], rtol=1e-4, atol=1e-6)
        np.testing.assert_allclose(to[s, :, :parts].double().cpu().numpy(), tmp[s, :, :parts], rtol=1e-4, atol=1e-5)
    assert ops.device_errors(0) == 0


@pytest.mark.parametrize("consumer", CONSUMERS)
@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
def test_constant_keys_give_mean_of_values(cflib, monkeypatch, dtype, consumer):
    """Known answer: identical K rows -> uniform softmax -> mean of the V rows."""
    import torch

    from cacheflow_b200 import ops

    _consumer(monkeypatch, dtype, consumer)

    rng = np.random.default_rng(7)
    ctx = [1, 16, 37, 600]
    H = Hkv = 2
    D = 128
    host, d = _setup(rng, dtype, H, Hkv, D, ctx)
    d["k"].copy_(d["k"][0:1, 0:1, 0:1, :].clone().expand_as(d["k"]))
    ops.paged_attention_v1(d["out"], d["q"], d["k"], d["v"], d["bt"], d["cl"], None, max(ctx))
    v = d["v"].double().cpu().numpy()
    tables = host[3]
    want = np.zeros((len(ctx), H, D))
    for s, c in enumerate(ctx):
        t = np.arange(c)
        rows = v[tables[s][t // 16], :, t % 16]  # [c, Hkv, D]
        want[s] = rows.mean(0)
    assert_close(as_f64(d["out"]), want, dtype, "constant K")


def test_one_hot_values_recover_weights(cflib, oracle_mod, monkeypatch):
    """V[t] = e_{t mod D}: output column d is the total weight of tokens t = d (mod D)."""
    import torch

    from cacheflow_b200 import ops

    rng = np.random.default_rng(11)
    D, ctx = 128, [100, 128, 300]
    host, d = _setup(rng, "f32", 1, 1, D, ctx)
    tables = host[3]
    vh = np.zeros_like(host[2])
    for s, c in enumerate(ctx):
        for t in range(c):
            vh[tables[s][t // 16], 0, t % 16, t % D] = 1.0
    d["v"].copy_(torch.from_numpy(vh))
    scale = 1.0 / math.sqrt(D)
    ops.paged_attention_v1(d["out"], d["q"], d["k"], d["v"], d["bt"], d["cl"], scale, max(ctx))
    got = as_f64(d["out"])
    q, k = host[0].astype(np.float64), host[1].astype(np.float64)
    for s, c in enumerate(ctx):
        t = np.arange(c)
        logits = k[tables[s][t // 16], 0, t % 16] @ q[s, 0] * np.float64(np.float32(scale))
        w = np.exp(logits - logits.max())
        w /= w.sum()
        want = np.bincount(t % D, weights=w, minlength=D)
        assert_close(got[s, 0], want, "f32", "one-hot V")
        assert abs(got[s, 0].sum() - 1.0) < 1e-5


@pytest.mark.parametrize("consumer", CONSUMERS)
def test_gqa_heads_with_equal_queries_agree(cflib, monkeypatch, consumer):
    import torch

    from cacheflow_b200 import ops

    _consumer(monkeypatch, "bf16", consumer)

    rng = np.random.default_rng(3)
    host, d = _setup(rng, "bf16", 8, 2, 128, [77, 1000])
    d["q"].copy_(d["q"][:, 0:1].clone().expand_as(d["q"]))  # every head asks the same question
    ops.paged_attention_v1(d["out"], d["q"], d["k"], d["v"], d["bt"], d["cl"], None, 1000)
    o = d["out"]
    for h in range(1, 4):
        assert torch.equal(o[:, h], o[:, 0])  # same kv head -> bitwise equal
        assert torch.equal(o[:, 4 + h], o[:, 4])


@pytest.mark.parametrize("consumer", CONSUMERS)
def test_empty_context_gives_zeros(cflib, monkeypatch, consumer):
    import torch

    from cacheflow_b200 import ops

    _consumer(monkeypatch, "f16", consumer)

    rng = np.random.default_rng(5)
    host, d = _setup(rng, "f16", 4, 4, 128, [0, 20, 0])
    d["out"].fill_(7.0)
    ops.paged_attention_v1(d["out"], d["q"], d["k"], d["v"], d["bt"], d["cl"], None, 20)
    assert torch.all(d["out"][0] == 0) and torch.all(d["out"][2] == 0)
    assert torch.all(d["out"][1] != 7.0)


@pytest.mark.parametrize("consumer", CONSUMERS)
def test_bad_block_id_is_recorded_not_read(cflib, monkeypatch, consumer):
    """An out-of-pool block id is skipped and flagged in the device error word."""
    from cacheflow_b200 import _lib, ops

    _consumer(monkeypatch, "bf16", consumer)

    rng = np.random.default_rng(9)
    host, d = _setup(rng, "bf16", 4, 4, 128, [40, 40])
    ops.device_errors(0, clear=True)
    pool = d["k"].shape[0]
    d["bt"][1, 1] = pool  # one past the end
    ops.paged_attention_v1(d["out"], d["q"], d["k"], d["v"], d["bt"], d["cl"], None, 40)
    bits = ops.device_errors(0, clear=True)
    assert bits & _lib.CF_DEVERR_BLOCK_ID
    assert ops.device_errors(0) == 0


def test_context_beyond_table_is_clamped_and_recorded(cflib):
    from cacheflow_b200 import _lib, ops

    rng = np.random.default_rng(12)
    host, d = _setup(rng, "f16", 2, 2, 128, [32, 32])
    ops.device_errors(0, clear=True)
    d["cl"][0] = 10_000  # table has 2 blocks
    ops.paged_attention_v1(d["out"], d["q"], d["k"], d["v"], d["bt"], d["cl"], None, 32)
    assert ops.device_errors(0, clear=True) & _lib.CF_DEVERR_CONTEXT_LEN


def test_unsupported_shapes_return_status(cflib):
    import torch

    from cacheflow_b200 import _lib, ops

    q = torch.zeros((1, 2, 96), dtype=torch.float16, device="cuda")
    k = torch.zeros((4, 2, 16, 96), dtype=torch.float16, device="cuda")
    bt = torch.zeros((1, 1), dtype=torch.int32, device="cuda")
    cl = torch.ones((1,), dtype=torch.int32, device="cuda")
    with pytest.raises(ops.CacheFlowError) as e:
        ops.paged_attention_v1(torch.empty_like(q), q, k, k, bt, cl, None, 1)
    assert e.value.status == _lib.CF_ERR_UNSUPPORTED


@pytest.mark.parametrize("consumer", CONSUMERS)
@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_garbage_past_context_does_not_leak(cflib, oracle_mod, monkeypatch, dtype, consumer):
    """Rows of the last block past the context may hold anything (here NaN)."""
    import torch

    from cacheflow_b200 import ops

    _consumer(monkeypatch, dtype, consumer)
    rng = np.random.default_rng(13)
    ctx = [1, 5, 17, 30, 100]
    host, d = _setup(rng, dtype, 8, 2, 128, ctx)
    q, k, v, tables, cl = host
    for s, c in enumerate(ctx):
        if c % 16:
            b = tables[s][c // 16]
            d["k"][b, :, c % 16:] = float("nan")
            d["v"][b, :, c % 16:] = float("nan")
    ops.paged_attention_v1(d["out"], d["q"], d["k"], d["v"], d["bt"], d["cl"], None, max(ctx))
    want = oracle_mod.paged_attention(q, k, v, tables, cl, 1 / math.sqrt(128), CODE[dtype])
    assert_close(as_f64(d["out"]), want, dtype, "NaN past context")
