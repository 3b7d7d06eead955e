"""The benchmark's JSON contract, checked without a GPU.

``bench.py --impl reference`` times the CPU restatement of the reference path
and must print one JSON line with the metric, the e2e block (no host-device
traffic) and a ``cpu_baseline`` describing itself.  The clock sampler's parser
decides whether a GPU run saw a throttle reason; it is fed a fake
``nvidia-smi`` CSV here.
"""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "2",
                        "--warmup", "0"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["unit"] == "voxels/s" and d["higher_is_better"] is True
    # the arm honours --steps / --warmup and prints our arm's config object
    assert d["value"] > 0 and d["steps"] == 2 and d["warmup"] == 0 and d["n_gpus"] == 1
    sys.path.insert(0, ROOT)
    import bench
    import __graft_entry__
    w = __graft_entry__.load_package().workloads.make_workload(2)
    assert d["config"] == bench.c2_config(w, 1, d["config"]["pairs"])
    assert d["config"]["pairs"] == 4679479  # valid (output, offset) pairs of the 256^3 workload's map
    assert d["config"]["workload"] and d["config"]["voxels"] > 0
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]


class _Running:
    """Stands in for the sampler's nvidia-smi process."""

    def poll(self):
        return None


def _summary(tmp_path, rows):
    sys.path.insert(0, ROOT)
    import bench
    path = tmp_path / "clocks.csv"
    path.write_text("".join(", ".join(r) + "\n" for r in rows))
    s = bench.ClockSampler(0)
    s.proc, s.path = _Running(), str(path)
    return s.summary()


def _row(sm, reasons=()):
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    flags = ["Active" if n in reasons else "Not Active" for n in names]
    return ["0", str(sm), "1965", "700.5", "0x0000000000000000"] + flags


def test_clock_summary_median_and_no_reason(tmp_path):
    out = _summary(tmp_path, [_row(1965), _row(1950), _row(1965)])
    assert out == {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": [], "samples": 3}


@pytest.mark.parametrize("reason", ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"])
def test_clock_summary_reports_each_throttle_reason(tmp_path, reason):
    out = _summary(tmp_path, [_row(1965), _row(1300, (reason,)), _row(1965)])
    assert out["reasons"] == [reason]
    assert out["samples"] == 3


def test_clock_summary_without_samples(tmp_path):
    out = _summary(tmp_path, [])
    assert out["samples"] == 0 and out["reasons"] == ["no samples"]
