"""CacheFlow's own host side driving the kernels end to end: its Scheduler,
BatchManager and BlockManager (reference sources, unchanged) produce each
step's SchedulerOutput and DecodeBatch; the C++ decode step of
include/cacheflow_b200_engine.hpp executes the block operations, stages the
rows and runs append + attention (oracle/ref_engine_driver.cpp).

A host mirror of the GPU and CPU pools follows the same block operations and
appends; every step, the device pools must equal the mirror bit for bit, and
every row's attention output must be within the bf16 tolerance of the oracle
computed on the mirror.  The run covers a prefill-only step (six prompts as
chunks), decode steps (fused append), a step with decode rows followed by two
new prompts (reshape + v1 + chunked prefill), and swap preemption (CacheFlow's
scheduler swaps the last running group out to the CPU pool and back in).
"""

import math

import numpy as np
import pytest

from cacheflow_b200.workloads import host_values
from helpers import as_f64, assert_close, to_dev

pytestmark = pytest.mark.gpu


def _host_bf16(t):
    return t.contiguous().cpu().view(__import__("torch").int16).numpy().view(np.uint16)


def test_cacheflow_scheduler_through_cpp_decode_step(cflib, oracle_mod):
    import torch

    from cacheflow_b200 import _lib, ops

    H, Hkv, D = 8, 2, 128
    ngpu, ncpu, mbps = 28, 256, 16
    rng = np.random.default_rng(101)
    mk = host_values((ngpu, Hkv, 16, D), "bf16", 0.5, rng)
    mv = host_values((ngpu, Hkv, 16, D), "bf16", 0.5, rng)
    mck = host_values((ncpu, Hkv, 16, D), "bf16", 0.5, rng)
    mcv = host_values((ncpu, Hkv, 16, D), "bf16", 0.5, rng)
    gk, gv = to_dev(mk, "bf16"), to_dev(mv, "bf16")

    def pinned(a):
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).pin_memory()

    ck, cv = pinned(mck), pinned(mcv)
    try:
        eng = oracle_mod.RefEngine(H, Hkv, D, _lib.CF_BF16, ngpu, ncpu, 16, 512, 512, mbps, gk.data_ptr(),
                                   gv.data_ptr(), ck.data_ptr(), cv.data_ptr())
    except FileNotFoundError:
        pytest.skip("oracle/_ref/libcf_ref_engine.so not built (make -C oracle ref)")
    stream = torch.cuda.current_stream().cuda_stream
    scale = 1.0 / math.sqrt(D)
    seen = {"prefill_only": 0, "mixed": 0, "fused": 0, "swaps_out": 0, "swaps_in": 0, "rows": 0}
    try:
        for r, p in enumerate([20, 37, 5, 64, 100, 17]):
            eng.add_request(r, p, 60)
        for step in range(24):
            if step == 3:  # two prompts arrive while six sequences decode
                eng.add_request(6, 33, 60)
                eng.add_request(7, 2, 60)
            c = eng.schedule(stream)
            swaps_out, swaps_in, copies = eng.block_ops(c)
            for s, d in swaps_out:
                mck[d], mcv[d] = mk[s], mv[s]
            for s, d in swaps_in:
                mk[d], mv[d] = mck[s], mcv[s]
            for s, d in copies:
                mk[d], mv[d] = mk[s], mv[s]
            n = c["rows"]
            if n:
                _, pos, tab = eng.rows(n)
                q_h = host_values((n, H, D), "bf16", 0.5, rng)
                kn_h = host_values((n, Hkv, D), "bf16", 0.5, rng)
                vn_h = host_values((n, Hkv, D), "bf16", 0.5, rng)
                q, kn, vn = to_dev(q_h, "bf16"), to_dev(kn_h, "bf16"), to_dev(vn_h, "bf16")
                out = torch.full((n, H, D), 9.0, dtype=torch.bfloat16, device="cuda")
                assert eng.attend(q.data_ptr(), out.data_ptr(), kn.data_ptr(), vn.data_ptr(), stream) == 0
                torch.cuda.synchronize()
                for i in range(n):
                    b = tab[i, pos[i] // 16]
                    mk[b, :, pos[i] % 16, :] = kn_h[i]
                    mv[b, :, pos[i] % 16, :] = vn_h[i]
                tables = np.ascontiguousarray(np.where(tab >= 0, tab, 0).astype(np.int32))
                want = oracle_mod.paged_attention(q_h, mk, mv, tables, (pos + 1).astype(np.int32), scale,
                                                  dtype_code=oracle_mod.BF16)
                assert_close(as_f64(out), want, "bf16", f"step {step}")
                seen["rows"] += n
                seen["fused"] += c["fused"]
                seen["prefill_only"] += int(c["chunks"] > 0 and c["decode_rows"] == 0)
                seen["mixed"] += int(c["chunks"] > 0 and c["decode_rows"] > 0)
            torch.cuda.synchronize()
            assert ops.device_errors(0) == 0, f"step {step}"
            assert np.array_equal(_host_bf16(gk), mk) and np.array_equal(_host_bf16(gv), mv), f"GPU pool, step {step}"
            assert np.array_equal(_host_bf16(ck), mck) and np.array_equal(_host_bf16(cv), mcv), f"CPU pool, step {step}"
            seen["swaps_out"] += c["swaps_out"]
            seen["swaps_in"] += c["swaps_in"]
            eng.finish_step(np.full(c["seqs"], 7, np.int32))
    finally:
        eng.close()
    assert seen["prefill_only"] >= 1 and seen["mixed"] >= 1 and seen["fused"] >= 10, seen
    assert seen["swaps_out"] >= 1 and seen["swaps_in"] >= 1, seen
