"""The operators inside CUDA graphs: a decode step (fused append + v1 split,
v2 + reduce, chunked prefill, cache ops) captured once after a warm-up call
(which makes the per-device, one-time kernel attribute settings) and replayed
gives the same results as eager calls."""

import numpy as np
import pytest

from cacheflow_b200.workloads import host_values
from helpers import random_tables, to_dev

pytestmark = pytest.mark.gpu


def test_decode_step_replays_in_a_graph(cflib):
    import torch

    from cacheflow_b200 import ops

    rng = np.random.default_rng(21)
    ctx = [1, 17, 700, 3000, 9000]
    S, H, Hkv, D = len(ctx), 32, 8, 128
    pool = sum((c + 15) // 16 for c in ctx) + 4
    tables = random_tables(rng, ctx, pool)
    k0 = host_values((pool, Hkv, 16, D), "bf16", 0.5, rng)
    v0 = host_values((pool, Hkv, 16, D), "bf16", 0.5, rng)
    cl = np.array(ctx, np.int32)
    pos = cl - 1
    slots = (tables[np.arange(S), pos // 16] * 16 + pos % 16).astype(np.int32)
    q = to_dev(host_values((S, H, D), "bf16", 0.5, rng), "bf16")
    nk = to_dev(host_values((S, Hkv, D), "bf16", 0.5, rng), "bf16")
    nv = to_dev(host_values((S, Hkv, D), "bf16", 0.5, rng), "bf16")
    bt, dcl, dsl = to_dev(tables), to_dev(cl), to_dev(slots)
    mctx = int(cl.max())
    P = ops.v2_num_partitions(mctx)

    def state():
        return to_dev(k0, "bf16"), to_dev(v0, "bf16")

    def step(k, v, out1, out2, es, ml, to, ws):
        ops.paged_attention_append_v1(out1, q, nk, nv, k, v, bt, dcl, dsl, None, mctx, workspace=ws)
        ops.paged_attention_v2(out2, es, ml, to, q, k, v, bt, dcl, None, mctx)

    def buffers():
        out1 = torch.empty((S, H, D), dtype=torch.bfloat16, device="cuda")
        out2 = torch.empty_like(out1)
        es = torch.empty((S, H, P), device="cuda")
        ml = torch.empty_like(es)
        to = torch.empty((S, H, P, D), device="cuda")
        n = ops.paged_attention_v1_workspace_size(q, torch.empty((pool, Hkv, 16, D)), bt, mctx)
        ws = torch.empty(max(n, 16), dtype=torch.uint8, device="cuda")
        return out1, out2, es, ml, to, ws

    # eager
    k_e, v_e = state()
    b_e = buffers()
    step(k_e, v_e, *b_e)
    torch.cuda.synchronize()
    # graph: warm-up call on a side stream, capture, then replay on fresh state
    k_g, v_g = state()
    b_g = buffers()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step(*state(), *buffers())
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step(k_g, v_g, *b_g)
    k_g.copy_(to_dev(k0, "bf16"))
    v_g.copy_(to_dev(v0, "bf16"))
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(k_g, k_e) and torch.equal(v_g, v_e)
    assert torch.equal(b_g[0], b_e[0]) and torch.equal(b_g[1], b_e[1])
    assert ops.device_errors(0) == 0


def test_prefill_and_cache_ops_replay_in_a_graph(cflib):
    import torch

    from cacheflow_b200 import ops

    rng = np.random.default_rng(22)
    chunks = [(0, 100), (500, 64), (37, 5)]
    ctx = [a + b for a, b in chunks]
    H, Hkv, D = 32, 8, 128
    pool = sum((c + 15) // 16 for c in ctx) + 8
    tables = random_tables(rng, ctx, pool)
    qs = np.zeros(len(chunks) + 1, np.int32)
    qs[1:] = np.cumsum([b for _, b in chunks])
    q = to_dev(host_values((int(qs[-1]), H, D), "bf16", 0.5, rng), "bf16")
    k = to_dev(host_values((pool, Hkv, 16, D), "bf16", 0.5, rng), "bf16")
    v = to_dev(host_values((pool, Hkv, 16, D), "bf16", 0.5, rng), "bf16")
    bt, dcl, dqs = to_dev(tables), to_dev(np.array(ctx, np.int32)), to_dev(qs)
    pairs = torch.tensor([[pool - 1, pool - 2]], dtype=torch.int64, device="cuda")
    zero_ids = torch.tensor([pool - 3], dtype=torch.int32, device="cuda")

    def step(out):
        ops.copy_blocks(k, v, pairs)
        ops.memset_blocks(k, zero_ids)
        ops.paged_prefill_attention(out, q, k, v, bt, dcl, dqs, None, 100)

    out_e = torch.empty_like(q)
    step(out_e)
    torch.cuda.synchronize()
    k_e = k.clone()
    out_g = torch.empty_like(q)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step(out_g)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out_g, out_e) and torch.equal(k, k_e)
    assert ops.device_errors(0) == 0
