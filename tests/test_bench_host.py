"""The benchmark's host logic, on the CPU: the clock record that decides whether a run is kept, and
the reference arm's JSON line (TriCast's CPU implementation on the host cores, rank 0 only)."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import bench

ROOT = Path(__file__).resolve().parent.parent


def test_clocks_summary_reports_throttle_reasons():
    # index, sm, max sm, power, active mask, hw_slowdown, hw_thermal, sw_thermal, sw_power_cap
    rows = [["0", "1965", "1965", "700", "0x0", "Not Active", "Not Active", "Not Active", "Not Active"],
            ["0", "1800", "1965", "990", "0x4", "Not Active", "Not Active", "Not Active", "Active"],
            ["0", "1965", "1965", "700", "0x0", "Not Active", "Not Active", "Not Active", "Not Active"]]
    s = bench.clocks_summary(rows)
    assert s["sm_mhz"] == 1965.0 and s["sm_max_mhz"] == 1965.0 and s["samples"] == 3
    assert s["reasons"] == ["sw_power_cap"]
    rows[0][6] = "Active"
    assert bench.clocks_summary(rows)["reasons"] == ["hw_thermal_slowdown", "sw_power_cap"]
    assert bench.clocks_summary([])["reasons"] == ["unsampled"]


def test_stats_ms():
    s = bench.stats_ms([3.0, 1.0, 2.0])
    assert s == {"median": 2.0, "mean": 2.0, "p99": 3.0, "n": 3}


def _run(args, env_extra=None):
    env = dict(os.environ, **(env_extra or {}))
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True, timeout=900,
                          env=env, cwd=ROOT)


def test_reference_arm_only_rank_zero_prints():
    r = _run(["--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "0"], {"RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0 and r.stdout.strip() == ""


def test_reference_arm_prints_one_json_line():
    r = _run(["--impl", "reference", "--steps", "1", "--warmup", "0"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "GMAC/s" and d["higher_is_better"] is True
    assert d["steps"] == 1 and d["warmup"] == 0 and d["value"] > 0
    assert d["metric"] == bench.METRIC and d["config"]["workload"] == bench.WORKLOAD
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "GMAC/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
