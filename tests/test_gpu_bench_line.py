"""GPU: bench.py's own arm prints one JSON line with the fields the bench
contract asks for (small shape, a few steps; the assembly / LM legs off)."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def test_bench_line_has_the_contract_fields():
    cmd = [sys.executable, str(ROOT / "bench.py"), "--steps", "4", "--warmup", "3",
           "--shape", "2048x65536x256x16", "--lm=", "--no-assembly", "--cpu-queries", "8"]
    res = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=900,
                         env={**os.environ, "PYTHONPATH": str(ROOT)})
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [l for l in res.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, res.stdout[-2000:]
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config", "e2e",
                "roofline", "cpu_baseline", "gpu_launches", "clocks"):
        assert key in d, key
    assert d["n_gpus"] == 1 and d["steps"] == 4 and d["warmup"] == 3
    assert d["value"] > 0 and d["ms_per_step"] > 0 and d["higher_is_better"] is True
    e2e = d["e2e"]
    assert e2e["value"] > 0 and e2e["h2d_bytes_per_step"] > 0 and e2e["d2h_bytes_per_step"] > 0
    roof = d["roofline"]
    assert roof["bound"] in ("tensor", "hbm") and 0 < roof["frac"] and roof["peak"] > 0
    assert abs(roof["frac"] - roof["achieved"] / roof["peak"]) < 1e-6
    cpu = d["cpu_baseline"]
    assert cpu["value"] > 0 and cpu["cores"] >= 1 and cpu["kind"] in ("port", "reference")
    assert d["gpu_launches"] > 0
    assert d["clocks"]["sm_max_mhz"] > 0
    assert d["device_status"] == 0
