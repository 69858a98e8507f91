"""bench.py's reference arm (CPU only): the JSON line the benchmark driver
reads, and the multi-rank rule (rank 0 alone runs it)."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _run(extra_env=None):
    env = dict(os.environ, **(extra_env or {}))
    return subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0"],
                          cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)


def test_reference_arm_prints_one_contract_line():
    sys.path.insert(0, str(ROOT))
    import bench

    r = _run()
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC and d["unit"] == bench.UNIT
    assert d["value"] > 0 and d["ms_per_step"] > 0
    # a step is the bounded sample that ran; value extrapolates it to a whole verify step
    assert d["extrapolated_ms_per_step"] > d["ms_per_step"]
    assert abs(d["value"] - 1e3 / d["extrapolated_ms_per_step"]) < 1e-9 * d["value"] + 1e-12
    assert (d["n_gpus"], d["steps"]) == (1, 1)
    assert d["warmup"] == 3  # fewer than 3 warm-up steps are raised to 3
    assert d["higher_is_better"] is True and d["scaling"] == "weak"
    assert d["config"]["workload"] == bench.workload_name()
    cpu = d["cpu_baseline"]
    assert cpu["value"] == d["value"] and cpu["kind"] == "port" and cpu["cores"] >= 1 and cpu["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_without_work():
    r = _run({"RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [ln for ln in r.stdout.splitlines() if ln.startswith("{")]


def test_clock_samples_summary():
    sys.path.insert(0, str(ROOT))
    import bench

    text = ("1965, 1965, Not Active, Not Active, Not Active, Not Active\n"
            "1905, 1965, Not Active, Not Active, Not Active, Active\n"
            "[N/A], 1965, Not Active, Not Active, Not Active, Not Active\n"
            "1950, 1965, Not Active, Not Active, Not Active, Not Active\n"
            "garbage\n")
    d = bench.parse_clock_samples(text)
    assert d == {"sm_mhz": 1950.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"]}
    assert bench.parse_clock_samples("") == {"sm_mhz": None, "sm_max_mhz": None, "reasons": []}
