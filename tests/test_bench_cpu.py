"""bench.py's reference arm on the host (CPU): one JSON line whose metric,
unit, direction and config are the GPU arm's, with the sample it timed in
cpu_baseline and a zero-copy e2e block."""

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_reference_arm_names_the_gpu_arms_workload():
    env = dict(os.environ, RANK="0", WORLD_SIZE="1", LOCAL_RANK="0")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "1"], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    name, m = bench.HEADLINE
    n, k = bench.LAYERS[name]
    assert line["impl"] == "reference"
    assert line["config"] == bench.arm_config(name, m, n, k, 1)
    assert line["metric"] == bench.METRIC and line["unit"] == "TFLOPS" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["cpu_baseline"]["value"] == line["value"]
    assert line["cpu_baseline"]["kind"] in ("reference", "port") and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"] == {"value": line["value"], "unit": "TFLOPS", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_the_headline_slices_evenly(world):
    name, m = bench.HEADLINE
    n, k = bench.LAYERS[name]
    cfg = bench.arm_config(name, m, n, k, world)
    assert cfg["n_per_gpu"] * world == n and cfg["n_per_gpu"] % 128 == 0
