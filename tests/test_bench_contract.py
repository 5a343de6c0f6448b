"""bench.py's reference arm (--impl reference) runs on the CPU: its JSON line
carries the keys the driver reads (metric, value, unit, steps, warm-up of at
least 3, ms_per_step, higher_is_better, config, the cpu_baseline description
and the e2e block with zero copy bytes), on the main arm's metric and
config."""
from __future__ import annotations

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "1"],
                         cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["unit"] == "rows/s" and line["higher_is_better"] is True
    # (warm-up is raised to the contract's minimum of 3 steps and reported so)
    assert line["steps"] == 1 and line["warmup"] == 3 and line["value"] > 0
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"] and cb["value"] == line["value"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert "workload" in line["config"]


def test_parallel_workload_generation_is_identical():
    """The bench generates config 4's 8192 rows on a thread pool; the values
    must equal the one-thread generator's, row for row."""
    import numpy as np
    sys.path.insert(0, ROOT)
    import __graft_entry__ as g
    pkg = g.load_package()
    rows = np.arange(37, 37 + 150)
    for name in ("c4_qwen2_sharded", "c3_batched_hetero"):
        a = pkg.workloads.make(name, rows=rows, V=3000)
        b = pkg.workloads.make_parallel(name, rows=rows, V=3000, threads=4, block=64)
        assert np.array_equal(a.logits, b.logits) and np.array_equal(a.params, b.params)
        assert np.array_equal(a.uniforms, b.uniforms) and np.array_equal(a.rows, b.rows)
        for f in ("hist_ids", "hist_off", "bias_ids", "bias_vals", "bias_off"):
            x, y = getattr(a, f), getattr(b, f)
            assert (x is None and y is None) or np.array_equal(x, y), f
