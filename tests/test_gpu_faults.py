"""The decode kernels' bounded pipeline waits, made to run out on purpose with
nothing in flight.

cf_testing_set_pipeline_faults shortens the wait limit to 1 ms and leaves the
first shared-memory stage of every warp unarmed: no copy is ever issued for
it and nothing arrives on its barrier, so the wait for it can only expire.
On a one-block context that stage is the only one, so no bulk copy is in
flight at any point.  The launch must come back promptly, record
CF_DEVERR_TIMEOUT, leave the output untouched, and the next normal call on
the same context must be correct.  No GPU fault or hang is involved: the
kernel returns on its own.
"""

import math
import time

import numpy as np
import pytest

from cacheflow_b200.workloads import host_values
from helpers import as_f64, assert_close, random_tables, to_dev, torch_dtype

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,H,Hkv,D", [("bf16", 8, 2, 128), ("f16", 4, 4, 64), ("f32", 4, 2, 128)])
def test_pipeline_wait_runs_out_and_the_next_call_is_correct(cflib, oracle_mod, dtype, H, Hkv, D):
    import torch

    from cacheflow_b200 import _lib, ops

    rng = np.random.default_rng(71)
    ctx = [5]  # one block: the unarmed stage is the only one
    pool = 4
    tables = random_tables(rng, ctx, pool)
    q_h = host_values((1, H, D), dtype, 0.5, rng)
    k_h = host_values((pool, Hkv, 16, D), dtype, 0.5, rng)
    v_h = host_values((pool, Hkv, 16, D), dtype, 0.5, rng)
    q, k, v = to_dev(q_h, dtype), to_dev(k_h, dtype), to_dev(v_h, dtype)
    bt, cl = to_dev(tables), to_dev(np.array(ctx, np.int32))
    scale = 1.0 / math.sqrt(D)
    sentinel = torch.full((1, H, D), 7.0, dtype=torch_dtype(dtype), device="cuda")
    out = sentinel.clone()
    ops.device_errors(0)  # start from a clear error word

    assert cflib.cf_testing_set_pipeline_faults(1_000_000, 1) == _lib.CF_OK
    try:
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        ops.paged_attention_v1(out, q, k, v, bt, cl, scale, max(ctx))
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
    finally:
        assert cflib.cf_testing_set_pipeline_faults(0, 0) == _lib.CF_OK
    errs = ops.device_errors(0)
    assert errs & _lib.CF_DEVERR_TIMEOUT, f"error word {errs:#x}"
    assert elapsed < 1.0, f"the expired wait took {elapsed:.3f} s"  # two 1 ms waits per CTA, not 2 s
    assert torch.equal(out, sentinel), "a CTA whose wait ran out wrote output"

    # the context is still usable and the next call is normal
    ops.paged_attention_v1(out, q, k, v, bt, cl, scale, max(ctx))
    torch.cuda.synchronize()
    assert ops.device_errors(0) == 0
    code = oracle_mod.BF16 if dtype == "bf16" else None
    want = oracle_mod.paged_attention(q_h, k_h, v_h, tables, np.array(ctx, np.int32), scale, dtype_code=code)
    assert_close(as_f64(out), want, dtype, "after the expired wait")


def test_pipeline_fault_hook_rejects_bad_values(cflib):
    from cacheflow_b200 import _lib

    assert cflib.cf_testing_set_pipeline_faults(-1, 0) == _lib.CF_ERR_INVALID_ARGUMENT
    assert cflib.cf_testing_set_pipeline_faults(0, 2) == _lib.CF_ERR_INVALID_ARGUMENT
    assert cflib.cf_testing_set_pipeline_faults(0, 0) == _lib.CF_OK
