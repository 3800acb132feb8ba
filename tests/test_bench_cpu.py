"""bench.py's reference arm keeps the line the driver reads, on CPU: one
JSON line with the arm's metric, unit, config and a cpu_baseline, e2e with
no host-device bytes (a small row count keeps it to seconds)."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_the_contract_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--steps", "2", "--warmup", "1", "--rows", "20000"],
                         capture_output=True, text=True, timeout=600, cwd=ROOT, check=True)
    lines = [ln for ln in out.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["value"] > 0 and d["unit"] == "rounds/s" and d["higher_is_better"] is True
    assert d["config"]["rows"] == 20000
    # the same run parameters and config as the GPU arm's line
    assert d["steps"] == 2 and d["warmup"] == 1
    sys.path.insert(0, ROOT)
    import bench

    bench.set_rows(20000)
    assert d["config"] == json.loads(json.dumps(bench.config(1)))
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] in ("port", "reference") and cb["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
