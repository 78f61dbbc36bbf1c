"""bench.py's reference arm (the oracle on the host cores) prints the one JSON
line of the benchmark contract; runs without a GPU."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_json_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1",
                        "--warmup", "3"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["value"] > 0 and d["unit"] == "TFLOP/s"
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 3
    assert d["higher_is_better"] is True
    assert d["config"]["workload"].startswith("c4_")
    assert d["cpu_baseline"]["kind"] in ("port", "reference") and d["cpu_baseline"]["cores"] >= 1
    assert d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def _bench_module():
    sys.path.insert(0, ROOT)
    import bench  # noqa: PLC0415
    return bench


def test_step_stats_median_spread_and_flag():
    bench = _bench_module()
    assert bench.step_stats([]) is None
    s = bench.step_stats([2.0, 2.0, 2.0, 2.0])
    assert s["median_ms"] == 2.0 and s["std_ms"] == 0.0 and s["over_5pct"] is False
    s = bench.step_stats([1.85, 1.86, 2.12, 2.13, 2.14])  # full clock, then power-capped
    assert s["median_ms"] == 2.12 and s["min_ms"] == 1.85 and s["max_ms"] == 2.14
    assert abs(s["rel_std"] - s["std_ms"] / 2.12) < 1e-12 and s["over_5pct"] is True


def test_rank_stats_slowest_rank_sets_the_time():
    bench = _bench_module()
    r = bench.rank_stats([20.0, 22.0, 21.0, 30.0], steps=10)
    assert r["min"] == 2.0 and r["max"] == 3.0 and r["ranks"] == 4
    assert abs(r["median"] - 2.15) < 1e-12


def test_clock_record_reports_the_capped_part():
    """A timed region that starts at full clock and settles under the power
    cap: the record keeps the median, the minimum, the share of samples more
    than 100 MHz below max and the reasons seen (gpu_idle dropped)."""
    bench = _bench_module()
    c = bench.ClockSampler.__new__(bench.ClockSampler)
    c.samples = [1965] * 3 + [1582] * 7
    c.reasons = {"sw_power_cap", "gpu_idle"}
    c.max_mhz = 1965
    c._t = None
    r = c.stop()
    assert r["sm_mhz"] == 1582 and r["sm_min_mhz"] == 1582 and r["sm_max_mhz"] == 1965
    assert abs(r["below_max_frac"] - 0.7) < 1e-12
    assert r["reasons"] == ["sw_power_cap"] and r["samples"] == 10
