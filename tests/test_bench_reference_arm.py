"""The reference arm of the benchmark (`bench.py --impl reference`) on the host cores: one JSON
line with the metric, unit and config of the GPU arm, its CPU baseline and its end-to-end value
(no host-device bytes). The driver runs this arm beside the GPU arm and divides their values, so
the line must parse and carry the same metric on the same workload."""

import json
import subprocess
import sys

from .common import GOLDEN

ROOT = GOLDEN.parent.parent


def test_reference_arm_prints_one_line_on_the_gpu_arms_metric():
    sys.path.insert(0, str(ROOT))
    import bench

    proc = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0"],
                          cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [ln for ln in proc.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, proc.stdout[-2000:]
    row = json.loads(lines[0])
    assert row["impl"] == "reference"
    assert row["metric"] == bench.METRIC and row["unit"] == "MB/s" and row["higher_is_better"] is True
    assert row["value"] > 0 and row["steps"] == 1 and row["n_gpus"] == 1
    assert row["config"]["same_config"] is True and row["config"]["window_tokens"] == bench.WINDOW
    cb = row["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == row["value"]
    assert cb["unit"] == "MB/s" and cb["sample"]
    e2e = row["e2e"]
    assert e2e == {"value": row["value"], "unit": "MB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
