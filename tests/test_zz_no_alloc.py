"""cf_paged_attention_v2_static_scratch: paged attention v2 for callers that
cannot allocate device memory (a host whose pool already owns all of the GPU's
memory, a decode thread that must not call cudaMalloc/cudaFree because they
can synchronise the device, a foreign-function host with raw pointers and no
allocator).  Its partition scratch lives in a fixed array inside the library.

Checked here through the C ABI against cf_paged_attention_v2 with
caller-allocated scratch, on two different calls in a row (the second call
must not be disturbed by what the first left in the shared array), plus the
rejection of a call whose scratch would not fit.  Kept in its own file, which
pytest collects last.
"""

import ctypes
import math

import numpy as np
import pytest

from cacheflow_b200.workloads import host_values
from helpers import as_f64, assert_close, random_tables, to_dev, torch_dtype

pytestmark = pytest.mark.gpu


def _call_pair(cflib, dtype, H, Hkv, D, ctx, seed):
    import torch

    from cacheflow_b200 import _lib, ops

    rng = np.random.default_rng(seed)
    S = len(ctx)
    pool = sum((c + 15) // 16 for c in ctx) + 5
    tables = random_tables(rng, ctx, pool)
    q_h = host_values((S, H, D), dtype, 0.5, rng)
    k_h = host_values((pool, Hkv, 16, D), dtype, 0.5, rng)
    v_h = host_values((pool, Hkv, 16, D), dtype, 0.5, rng)
    q, k, v = to_dev(q_h, dtype), to_dev(k_h, dtype), to_dev(v_h, dtype)
    bt, cl = to_dev(tables), to_dev(np.array(ctx, np.int32))
    out_static = torch.full((S, H, D), 9.0, dtype=torch_dtype(dtype), device="cuda")
    out_ref = torch.empty_like(out_static)
    scale = 1.0 / math.sqrt(D)
    stream = torch.cuda.current_stream().cuda_stream

    # the existing entry point, scratch allocated by the caller
    P = ops.v2_num_partitions(max(ctx))
    es = torch.empty((S, H, P), device="cuda")
    ml = torch.empty_like(es)
    to = torch.empty((S, H, P, D), device="cuda")
    p_ref = ops._attention_params(out_ref, q, k, v, bt, cl, scale, max(ctx))
    assert cflib.cf_paged_attention_v2(ctypes.byref(p_ref), es.data_ptr(), ml.data_ptr(), to.data_ptr(), P,
                                       stream) == _lib.CF_OK

    # the no-allocation entry point: inputs and output only
    p = ops._attention_params(out_static, q, k, v, bt, cl, scale, max(ctx))
    assert cflib.cf_paged_attention_v2_static_scratch(ctypes.byref(p), stream) == _lib.CF_OK
    torch.cuda.synchronize()
    assert ops.device_errors(0) == 0
    # the same kernels on the same inputs: bit-identical, not just close
    assert torch.equal(out_static, out_ref), "static-scratch v2 differs from v2 with caller scratch"
    # and both within the attention tolerance of the oracle
    from oracle import oracle

    code = oracle.BF16 if dtype == "bf16" else None  # f16 arrays carry their own dtype
    want = oracle.paged_attention(q_h, k_h, v_h, tables, np.array(ctx, np.int32), scale, dtype_code=code)
    assert_close(as_f64(out_static), want, dtype, "static-scratch v2 vs oracle")


def test_static_scratch_matches_v2_on_two_calls_in_a_row(cflib):
    # first call: long GQA contexts (many partitions)
    _call_pair(cflib, "bf16", 32, 8, 128, [5, 600, 3000, 4097, 1, 2500], seed=31)
    # second call: other shapes, fewer rows -- stale scratch from the first
    # call must not leak into it
    _call_pair(cflib, "f16", 8, 8, 64, [17, 9000, 513], seed=32)


def test_static_scratch_rejects_calls_that_do_not_fit(cflib):
    from cacheflow_b200 import _lib

    p = _lib.AttentionParams()
    p.num_seqs, p.num_heads, p.num_kv_heads, p.head_dim, p.block_size = 64, 64, 8, 128, 16
    p.max_context_len, p.max_blocks_per_seq = 32768, 2048
    p.dtype = _lib.CF_BF16
    # 64 * 64 * 64 partitions * 130 floats = 136 MB > 16 MiB: refused, nothing launched
    assert cflib.cf_paged_attention_v2_static_scratch(ctypes.byref(p), None) == _lib.CF_ERR_WORKSPACE
    assert cflib.cf_paged_attention_v2_static_scratch(None, None) == _lib.CF_ERR_INVALID_ARGUMENT
    # shapes the kernels do not take are refused as unsupported before any
    # size arithmetic, however large
    p.head_dim = 96
    assert cflib.cf_paged_attention_v2_static_scratch(ctypes.byref(p), None) == _lib.CF_ERR_UNSUPPORTED
    p.head_dim, p.num_seqs, p.num_heads = 128, 1 << 30, 1 << 30
    assert cflib.cf_paged_attention_v2_static_scratch(ctypes.byref(p), None) == _lib.CF_ERR_UNSUPPORTED
