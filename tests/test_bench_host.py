"""Host-side pieces of bench.py that decide whether a measurement stands:
the clock record (throttle reasons that reject a run) and the roofline inputs."""
import importlib.util
import json
import os

from conftest import ROOT


def bench():
    spec = importlib.util.spec_from_file_location("bench_module", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_clock_summary_reports_median_and_active_reasons():
    b = bench()
    lines = [
        "0, 1965, 1965, 700.5, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
        "0, 1800, 1965, 998.1, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "0, 1700, 1965, 999.0, 0x0000000000000008, Active, Not Active, Not Active, Active",
        "1, 900, 1965, 300.0, 0x0000000000000040, Not Active, Active, Not Active, Not Active",  # another GPU
        "0, [N/A], 1965, 0, 0x0, Not Active, Not Active, Not Active, Not Active",              # unreadable
        "garbage",
    ]
    s = b.ClockSampler.summarise(lines, 0)
    assert s["samples"] == 3
    assert s["sm_mhz"] == 1800.0
    assert s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["hw_slowdown", "sw_power_cap"]
    assert b.ClockSampler.summarise([], 0) == {"sm_mhz": None, "sm_max_mhz": None, "samples": 0, "reasons": []}


def test_roofline_inputs_are_present_and_consistent():
    b = bench()
    peak, source = b.measured_peaks()
    assert peak > 1000 and source
    t = b.measured_traffic()
    assert t is not None, "profiles/traffic.json missing"
    with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
        assert json.load(f) == t
    # the recorded ratio is the capture's own read + write over algorithmic bytes
    r = t["decode_step_ratio"]
    assert abs((r["dram_read"] + r["dram_write"]) / r["algorithmic"] - r["ratio"]) < 1e-3
    g = t["gemv_gate_up_8b"]
    assert 0.99 < (g["dram_read"] + g["dram_write"]) / g["algorithmic"] < 1.05


def test_gemv_cpu_baseline_reports_each_thread_count():
    b = bench()
    r = b.gemv_cpu_baseline(rows=64, cols=256, threads=(1, 2), seconds=0.01)
    assert r["unit"] == "GB/s" and r["shape"] == "64x256" and r["kind"] == "port"
    assert r["threads_1"] > 0 and r["threads_2"] > 0
