"""bench.py's reference arm runs on the host cores alone (the reference's
own moe_layer, compiled from its sources, or the restatement where it is
not built): its JSON line carries the fields the driver reads."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KEYS = ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
        "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
        "cpu_baseline", "e2e")


@pytest.mark.parametrize("workload", ["kimi", "k3"])
def test_reference_arm_line(workload):
    cmd = [sys.executable, "bench.py", "--impl", "reference", "--workload", workload,
           "--steps", "1", "--warmup", "3", "--cpu-budget", "2"]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600,
                       env=dict(os.environ, CUDA_VISIBLE_DEVICES=""))
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    for k in KEYS:
        assert k in line, k
    assert line["impl"] == "reference"
    assert line["value"] > 0 and line["higher_is_better"] is True
    assert line["config"]["workload"] in ("kimi_linear_48b_moe_decode",
                                          "k3_class_moe_layer_decode")
    cb = line["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == line["value"] and cb["unit"] == line["unit"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
