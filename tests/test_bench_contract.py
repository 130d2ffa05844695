"""The benchmark's reference arm prints the driver's JSON contract on a host without a GPU.

`bench.py --impl reference` times the reference's CPU arithmetic for each config's path on
the host cores; here each config runs one warm-up and one timed step and its single JSON
line is checked for the keys the driver reads (metric, value, unit, impl, the CPU baseline
description and an `e2e` block with no host/device traffic), for the same ``config`` as
this build's own line, and for an ``ms_per_step`` that is the time actually spent per step
(so ``steps x ms_per_step`` fits in the run).
"""

import json
import os
import subprocess
import sys
import time

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("config", ["window", "indexer", "prefill", "decode", "train", "candidates", "compressor", "normrope"])
def test_reference_arm_json_line(config):
    cmd = [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--config", config,
           "--steps", "1", "--warmup", "1", "--cpu-sample", "64"]
    t0 = time.time()
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, cwd=ROOT)
    wall = time.time() - t0
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert isinstance(d["metric"], str) and d["unit"] and d["value"] > 0
    assert d["higher_is_better"] is True and d["steps"] == 1 and d["warmup"] == 1
    assert d["config"]["workload"]
    import bench
    assert d["config"] == bench.CONFIGS[config](1), "the reference arm must report this build's config"
    assert d["steps"] * d["ms_per_step"] / 1e3 <= wall, "ms_per_step must be the time of the work done"
    cb = d["cpu_baseline"]
    assert cb["value"] == pytest.approx(d["value"]) and cb["unit"] == d["unit"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    e = d["e2e"]
    assert e["value"] == pytest.approx(d["value"]) and e["unit"] == d["unit"]
    assert e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0
