"""CPU checks of bench.py's contract pieces that need no GPU: the metric
names, and the reference arm's JSON line on the CPU-runnable workload."""
from __future__ import annotations

import json
import os
import subprocess
import sys

from conftest import ROOT


def test_metric_names():
    import bench
    import workloads

    assert bench.metric_name(workloads.WORKLOADS["flux"]) == bench.METRIC
    assert "M=N=4608,d=128,H=24" in bench.METRIC
    cross = bench.metric_name(workloads.WORKLOADS["cross"])
    assert "M=4096,N=512,d=128,H=48" in cross and cross != bench.METRIC


def test_reference_arm_line(oracle_built):
    out = subprocess.run(
        [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload",
         "cpu_case", "--steps", "2", "--warmup", "3", "--cpu-rows-per-step", "8"],
        capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "TFLOP/s" and d["higher_is_better"] is True
    assert d["steps"] == 2 and d["warmup"] == 3 and d["value"] > 0
    assert d["e2e"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] in ("reference", "port") and d["cpu_baseline"]["cores"] >= 1
