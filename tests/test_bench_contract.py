"""The bench line's keys, checked on the CPU through the reference arm
(`bench.py --impl reference` times CacheFlow's CPU decode step and needs no
GPU): the same JSON shape the GPU arm prints."""

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "1"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["n_gpus"] == 1 and d["warmup"] >= 3
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert d["config"]["workload"] == "llama3_70b_sharded" and d["scaling"] == "strong"
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_cpu_samples_cut_contexts_not_rows():
    """The CPU baselines' bounded samples keep their rows (the reference step
    spreads rows over its threads) and cut each context to its first tokens;
    the block ids are renumbered into a compact pool."""
    import numpy as np

    sys.path.insert(0, str(ROOT))
    import bench
    from cacheflow_b200 import workloads

    w = workloads.make("llama3_70b_sharded")
    ctx, tables, pool = bench.reference_sample(w, 16, 100)
    assert len(ctx) == 16 and int(ctx.max()) <= 100 and np.all(ctx == np.minimum(w.context_lens[:16], 100))
    nblk = (ctx.astype(np.int64) + 15) // 16
    used = np.concatenate([tables[i, :nblk[i]] for i in range(len(ctx))])
    assert pool == len(np.unique(used)) and used.min() == 0 and used.max() == pool - 1

    r = bench.cpu_port_baseline(workloads.make("cpu_decode_fp32"), budget_s=0.2)
    assert r["kind"] == "port" and r["value"] > 0 and r["value_one_thread"] > 0 and r["cores"] >= 1
