"""bench.py's command-line contract, on CPU.

The reference arm times the reference's CPU GEMM (or its port) and must print
one JSON line with the same metric, config and keys as the GPU arm; under a
multi-rank launch only rank 0 prints.  The GPU arm has no CPU fallback: without
a GPU it must fail, not print a number.
"""
from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench(*args, env=None, timeout=240):
    e = dict(os.environ)
    e.update(env or {})
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], capture_output=True, text=True,
                          timeout=timeout, env=e, cwd=ROOT)


@pytest.mark.parametrize("config", ["2", "4"])
def test_reference_arm_prints_one_complete_line(config):
    r = _bench("--impl", "reference", "--config", config, "--steps", "1", "--warmup", "0", "--cpu-seconds", "1")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    import bench

    assert d["impl"] == "reference" and d["metric"] == bench.METRIC and d["unit"] == "TFLOP/s"
    assert d["value"] > 0 and d["higher_is_better"] is True and d["n_gpus"] == 1
    assert d["steps"] == 1 and d["warmup"] == 0 and d["ms_per_step"] > 0
    assert d["config"]["workload"] == bench.CONFIGS[int(config)]["name"]
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["cores"] >= 1 and cb["kind"] in ("reference", "port") and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_prints_nothing_on_other_ranks():
    r = _bench("--impl", "reference", "--steps", "1", "--warmup", "0", env={"RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0 and r.stdout.strip() == ""


def test_gpu_arm_fails_without_a_gpu():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    r = _bench("--steps", "1", "--warmup", "0", "--no-cpu-baseline", timeout=120)
    assert r.returncode != 0
    assert "value" not in r.stdout
