"""The benchmark's CPU-side pieces: the calculator's floors and the reference
arm's JSON line (its CPU path runs here on the whole headline workload)."""

import json
import subprocess
import sys
from pathlib import Path

from ace_kernels_b200 import calculator as calc
from ace_kernels_b200 import workloads as wl

ROOT = Path(__file__).resolve().parents[1]


def test_calculator_matches_the_reference_formulas() -> None:
    w = wl.WORKLOADS["c2_soft_2x3x128c"]
    nb = calc.ideal_bytes(w.input_bytes(), w.target_bytes(), "fwd_bwd")
    assert nb == 218_103_808 == w.ideal_bytes()
    assert calc.ideal_bytes(w.input_bytes(), w.target_bytes(), "fwd") == 83_886_080
    assert abs(calc.bandwidth_floor_ms(nb, 6548.5) * 1e3 - 33.306) < 1e-2
    assert calc.launch_floor_ms(3) == 0.015  # the reference's 5 us per launch
    assert abs(calc.effective_gbps(nb, 0.05) - 4362.08) < 1e-1


def test_reference_arm_line() -> None:
    out = subprocess.run(
        [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
         "--warmup", "0"], capture_output=True, text=True, timeout=600, cwd=ROOT,
    )
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["config"]["workload"] == "c2_soft_2x3x128c"
    assert line["config"]["shape"] == [2, 3, 128, 128, 128]
    assert line["cpu_baseline"]["kind"] == "port"
    assert line["e2e"]["h2d_bytes_per_step"] == 0
    assert "whole workload" in line["cpu_baseline"]["sample"]
    assert line["value"] > 0 and line["steps"] == 1
