"""The benchmark script's host-side contract (no GPU): the reference arm's
`unavailable` line, the clock-sample summary, and the synthetic workload."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_reference_arm_prints_unavailable_and_exits_zero():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--gpus", "2", "--steps", "3",
                        "--warmup", "3"], cwd=ROOT, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unavailable"] and d["n_gpus"] == 2


def test_clock_summary_median_and_reasons():
    lines = [
        "1800, 1965, 900.1, 0x4, Not Active, Not Active, Not Active, Active",
        "1850, 1965, 950.0, 0x4, Not Active, Not Active, Not Active, Active",
        "1900, 1965, 990.0, 0x0, Not Active, Not Active, Not Active, Not Active",
        "garbage line",
        "[N/A], 1965, 1.0, 0x0, Not Active, Not Active, Not Active, Not Active",
    ]
    c = bench.summarize_clocks(lines)
    assert c["sm_mhz"] == 1850 and c["sm_max_mhz"] == 1965 and c["samples"] == 3
    assert c["reasons"] == ["sw_power_cap"]
    hot = bench.summarize_clocks(["1200, 1965, 700, 0x40, Not Active, Active, Not Active, Not Active"])
    assert hot["reasons"] == ["hw_thermal_slowdown"]


def test_workload_shape_and_determinism():
    p1, o1, a1 = bench.build_workload(64, 1000, 128256, 200.0)
    p2, o2, a2 = bench.build_workload(64, 1000, 128256, 200.0)
    assert p1 == p2 and o1 == o2 and a1 == a2               # every data-parallel rank serves this stream
    assert all(128 <= len(p) <= 2048 for p in p1) and all(64 <= o <= 512 for o in o1)
    assert all(0 <= t < 128256 for p in p1 for t in p)
    assert all(b >= a for a, b in zip(a1, a1[1:]))           # Poisson arrivals are increasing
