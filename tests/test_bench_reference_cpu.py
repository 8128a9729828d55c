"""`bench.py --impl reference` (the reference's CPU path, here the C port of
it) prints one JSON line with the same metric, unit, direction and workload
as the CUDA arm, its e2e block with no host-device copies, and the
cpu_baseline that describes it.  Runs on the CPU in a few seconds.
"""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_json_contract():
    res = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1"],
                         cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, res.stdout[-2000:]
    d = json.loads(lines[0])
    sys.path.insert(0, str(ROOT))
    import bench

    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC
    assert d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 1
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["config"]["workload"].startswith("config 3: paged GQA decode with fused append")
    assert d["config"]["tokens_in_cache"] == 309_371 and d["config"]["pages"] == 19_369
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["unit"] == "GB/s" and cb["kind"] == "port" and cb["cores"] >= 1
    assert cb["sample"]
    e2e = d["e2e"]
    assert e2e == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
