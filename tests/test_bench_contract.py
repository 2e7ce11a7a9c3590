"""bench.py's command-line contract, checked on the CPU through its reference
arm (the NumPy restatement of the reference path timed on the host cores):
one JSON line with the metric, the config it names and the e2e / cpu_baseline
objects; argument errors exit with status 2 before any work.
"""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(*args, timeout=300, env=None):
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT,
                          capture_output=True, text=True, timeout=timeout,
                          env=None if env is None else {**os.environ, **env})


def _line(res):
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, res.stdout
    return json.loads(lines[0])


def test_reference_arm_line():
    d = _line(_run("--impl", "reference", "--workload", "c1_op", "--steps", "2", "--warmup", "3",
                   "--cpu-queries", "8"))
    assert d["impl"] == "reference"
    assert d["metric"] == "fused score+top-k retrieval queries/s"
    assert d["unit"] == "queries/s" and d["higher_is_better"] is True
    assert d["steps"] == 2 and d["warmup"] == 3 and d["n_gpus"] == 1
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["config"]["workload"] == "c1_op"
    assert (d["config"]["M"], d["config"]["N"], d["config"]["d"], d["config"]["k"]) == \
        (2048, 16384, 128, 16)
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert d["jax"]  # the probe of the reference's own runtime is recorded


def test_reference_arm_stays_within_its_budget():
    """The default 320 timed steps: each step scores a pool slice sized to the
    budget, and the time is scaled to the full pool."""
    import time

    t0 = time.time()
    d = _line(_run("--impl", "reference", "--workload", "c1_op", "--warmup", "3",
                   "--cpu-queries", "8", "--reference-budget-s", "6"))
    assert d["steps"] == 320
    assert 0 < d["config"]["sample_pool_rows"] <= 16384
    assert time.time() - t0 < 120


def test_shape_override_names_the_workload_by_its_sizes():
    d = _line(_run("--impl", "reference", "--shape", "300x5000x64x32", "--steps", "1",
                   "--warmup", "3", "--cpu-queries", "4"))
    cfg = d["config"]
    assert cfg["workload"] == "shape_300x5000x64x32"
    assert (cfg["M"], cfg["N"], cfg["d"], cfg["k"]) == (300, 5000, 64, 32)


def test_reference_arm_other_ranks_exit_quietly():
    """Under torchrun with N > 1 only rank 0 times and prints the reference arm."""
    res = _run("--impl", "reference", "--gpus", "2", "--workload", "c1_op", "--steps", "1",
               "--warmup", "3", "--cpu-queries", "4",
               env={"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"})
    assert res.returncode == 0, res.stderr[-1000:]
    assert not [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
    d = _line(_run("--impl", "reference", "--gpus", "2", "--workload", "c1_op", "--steps", "1",
                   "--warmup", "3", "--cpu-queries", "4",
                   env={"RANK": "0", "LOCAL_RANK": "0", "WORLD_SIZE": "2"}))
    assert d["n_gpus"] == 2 and d["impl"] == "reference"


@pytest.mark.parametrize("args", [
    ("--warmup", "2"),
    ("--shape", "16384x262144x4096"),
    ("--shape", "axbxcxd"),
    ("--workload", "no_such_workload"),
])
def test_argument_errors_exit_2(args):
    res = _run("--impl", "reference", *args, timeout=120)
    assert res.returncode == 2, (res.returncode, res.stderr[-500:])
