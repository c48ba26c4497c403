"""bench.py's host-side helpers on the CPU: the clock summary that decides whether a run
is kept (throttle reasons, median clock), the GPU naming for nvidia-smi, and the
whole-job rate."""

import pytest

import bench
from conftest import gpu_available


def _row(idx, sm, mx, *reasons):
    active = ["Active" if r else "Not Active" for r in reasons]
    return [str(idx), str(sm), str(mx), "700.0", "0x4"] + active


def test_clock_summary():
    c = bench.ClockSampler("GPU-x")
    assert c.summary()["reasons"] == ["unsampled"]
    c.rows = [_row(3, 1480, 1965, 0, 0, 0, 1), _row(3, 1500, 1965, 0, 0, 0, 1), _row(3, 1965, 1965, 0, 0, 0, 0),
              ["3", "[N/A]", "1965", "0", "0x0", "Not Active", "Not Active", "Not Active", "Not Active"]]
    s = c.summary()
    assert s["sm_mhz"] == 1500.0 and s["sm_max_mhz"] == 1965.0 and s["samples"] == 4
    assert s["reasons"] == ["sw_power_cap"] and s["nvidia_smi_index"] == "3"
    c.rows.append(_row(3, 900, 1965, 1, 0, 1, 0))  # a slowdown anywhere in the region is reported
    assert c.summary()["reasons"] == ["hw_slowdown", "sw_power_cap", "sw_thermal_slowdown"]


@pytest.mark.skipif(gpu_available(), reason="checks the fallback without a GPU")
def test_smi_id_falls_back_to_the_index():
    assert bench.smi_id(2) == "2"


def test_job_rate():
    # 8 ranks x 128 clips x 60 s x 10 steps over the slowest rank's 1.875 s
    assert bench.job_rate(8, 128, 60.0, 10, 1875.0) == pytest.approx(8 * 128 * 60.0 * 10 / 1.875)


def test_window_flops_is_the_published_formula():
    import synth

    cfg = synth.MODEL_CONFIG
    for S, G in [(1, 0), (684, 380), (370, 3), (0, 1)]:
        assert bench.window_flops(cfg, S, G) == 197_615_616 * S + 63_488 * S * S + 1_048_576 * G


def test_run_flops_over_the_planned_schedule(checkpoint_dir):
    """A 60 s clip: 3 offline windows, 333.0 GFLOP; 250 ultra-low-latency windows,
    14 600.6 GFLOP (G counts every newly embedded row, look-ahead included, since each
    streaming chunk is embedded whole); identical lengths are planned once."""
    off = bench.run_flops(checkpoint_dir, [960_000] * 3, "offline")
    assert round(off / 3 / 1e9, 1) == 333.0
    ultra = bench.run_flops(checkpoint_dir, [960_000], "ultra_low_latency")
    assert round(ultra / 1e9, 1) == 14600.6
