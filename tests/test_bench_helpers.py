"""bench.py's host-side helpers on the CPU: clock windows, roofline choice, denominators, configs."""

import json

import pytest

import bench


def test_fp8_denominator_is_twice_the_measured_bf16():
    peaks = {"bf16_tflops": 1630.8, "bf16_tflops_sustained": 1379.6, "hbm_gbs": 6544.7}
    burst, src = bench.fp8_peak(peaks, "measured", False)
    sustained, src_s = bench.fp8_peak(peaks, "measured", True)
    assert burst == pytest.approx(3261.6) and "bf16_tflops" in src
    assert sustained == pytest.approx(2759.2) and "sustained" in src_s


def test_roofline_entry_picks_the_bound_by_intensity():
    peaks = {"bf16_tflops": 1630.8, "hbm_gbs": 6544.7}
    # M = 16 x 28672 x 8192: ~31 FLOP/B, HBM-bound.
    m, n, k = 16, 28672, 8192
    flops, nbytes = 2.0 * m * n * k, float(m * k + n * k + (m + n) * (k // 32) + 2 * m * n)
    e = bench.roofline_entry(flops, nbytes, 0.040, peaks, "measured")
    assert e["roofline"]["bound"] == "hbm" and e["roofline"]["unit"] == "GB/s"
    assert e["roofline"]["frac"] == pytest.approx(nbytes / 40e-6 / 1e9 / 6544.7)
    # 4096^3: far above the ridge, tensor-bound.
    m = n = k = 4096
    flops, nbytes = 2.0 * m * n * k, float(m * k + n * k + (m + n) * (k // 32) + 2 * m * n)
    e = bench.roofline_entry(flops, nbytes, 0.050, peaks, "measured")
    assert e["roofline"]["bound"] == "tensor" and e["roofline"]["peak"] == pytest.approx(3261.6)


def test_both_arms_emit_the_same_config():
    a = bench.workload_config(16384, 16384, 16384, 1, "square")
    b = bench.workload_config(16384, 16384, 16384, 1, "square")
    assert a == b and a["workload"] == "mxfp8_fprop_m16384_n16384_k16384" and "l2" in a
    assert bench.workload_config(16384, 16384, 16384, 8, "square")["parallelism"] == "n-shard8"
    json.dumps(a)


def test_clock_sampler_summarises_only_the_timed_window():
    s = bench.ClockSampler(0)
    s.samples = [(0.5, 1965.0, 1965.0, 300.0, 0), (1.1, 1400.0, 1965.0, 900.0, 0x4), (1.2, 1300.0, 1965.0, 990.0, 0x4),
                 (2.5, 1965.0, 1965.0, 250.0, 0)]
    s.window = [1.0, 1.3]
    out = s.stop()
    assert out["samples"] == 2 and out["sm_mhz"] == pytest.approx(1350.0) and out["sm_mhz_min"] == 1300.0
    assert out["reasons"] == ["sw_power_cap"] and out["power_w_max"] == 990.0
    assert out["window_ms"] == pytest.approx(300.0)


def test_clock_sampler_reports_an_empty_window():
    s = bench.ClockSampler(0)
    s.window = [1.0, 1.01]
    out = s.stop()
    assert out["samples"] == 0 and out["sm_mhz"] is None


def test_side_configurations_cover_the_baseline_shapes():
    names = {g[0] for g in bench.SIDE_GEMMS}
    assert {"mxfp8_fprop_m4096_n4096_k4096", "mxfp8_fprop_m8192_n28672_k8192", "mxfp8_fprop_m128_n28672_k8192",
            "mxfp8_fprop_m16_n28672_k8192"} <= names
    # Only the shape whose operands fit in the L2 rotates operand sets.
    assert [g[0] for g in bench.SIDE_GEMMS if g[6] == "rotate"] == ["mxfp8_fprop_m4096_n4096_k4096"]
