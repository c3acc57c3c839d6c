"""bench.py's reference arm on the CPU: the JSON line the driver reads, and the rank behaviour under a launcher.

The reference arm times the reference's CPU semantics (the oracle port) on the host cores, so it runs here without a
GPU; the GPU arm's line is checked by running it on a B200."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(env_extra=None, *args):
    env = dict(os.environ)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                           "--warmup", "3", *args], capture_output=True, text=True, env=env, cwd=ROOT, timeout=600)


@pytest.fixture(scope="module")
def reference_line():
    r = _run()
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout  # exactly one JSON line on stdout
    return json.loads(lines[0])


def test_reference_arm_json_contract(reference_line):
    d = reference_line
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 3
    assert d["higher_is_better"] is True and d["data"] == "synthetic"
    assert d["config"]["workload"] == "sd15-linear-sweep+attention-blocks"
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["unit"] == d["unit"] and cb["cores"] >= 1
    assert cb["kind"] in ("port", "reference") and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_matches_the_gpu_arm_metric(reference_line):
    import bench
    assert reference_line["metric"] == bench.METRIC  # the same metric name as the GPU arm's line
    assert reference_line["unit"] == "TFLOP/s"
    assert reference_line["config"] == json.loads(json.dumps(bench.hotpath_config(1)))  # the GPU arm's config
    assert "whole 70-op step" in reference_line["cpu_baseline"]["sample"]


def test_reference_arm_other_ranks_exit_without_work():
    r = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""
