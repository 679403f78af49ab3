"""Host-side pieces of bench.py that decide what a bench line reports: the bf16
parity counts, the clock-sample summary that screens throttled runs, and the
roofline denominators. No GPU needed."""

import json
import os

import numpy as np

import bench


def _bf16(values):
    a = np.asarray(values, dtype=np.float32)
    return (a.view(np.uint32) >> 16).astype(np.uint16)


def test_bf16_parity_counts():
    want = _bf16([1.0, -2.0, 0.0, 3.0, 1e-30])
    got = want.copy()
    r = bench.bf16_parity(got, want)
    assert r == {"n": 5, "max_abs": 0.0, "bit_mismatch": 0, "over_1ulp": 0,
                 "max_abs_where_over_1ulp": 0.0}
    got[0] += 1                      # one bf16 ulp above 1.0
    got[2] = 0x8000                  # -0 counts as +0
    r = bench.bf16_parity(got, want)
    assert r["bit_mismatch"] == 1 and r["over_1ulp"] == 0
    assert r["max_abs"] == 2.0 ** -7
    got[4] = want[4] | 0x8000        # sign flip of a tiny value: many ulps, tiny error
    r = bench.bf16_parity(got, want)
    assert r["over_1ulp"] == 1 and r["max_abs_where_over_1ulp"] < 1e-29


def test_clock_summary_reports_median_and_reasons():
    s = bench.ClockSampler(0)
    assert s.summary()["reasons"] == ["unsampled"]
    row = lambda mhz, power_cap, thermal: [  # noqa: E731
        "0", str(mhz), "1965", "900.0", "0x4", "Not Active", "Not Active",
        "Active" if thermal else "Not Active", "Active" if power_cap else "Not Active"]
    s.samples = [row(1800, True, False), row(1900, False, False), row(1850, True, False)]
    r = s.summary()
    assert r == {"sm_mhz": 1850.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"],
                 "samples": 3}
    s.samples.append(row(1200, False, True))
    assert "sw_thermal_slowdown" in s.summary()["reasons"]


def test_peaks_come_from_the_measured_file():
    path = os.path.join(bench.REPO, "MEASURED_PEAKS.json")
    if not os.path.exists(path):
        v, src = bench.load_peaks("hbm_gbs")
        assert src == "fallback" and v == bench.FALLBACK_HBM_GBS
        return
    with open(path) as f:
        peaks = json.load(f)
    for key in ("hbm_gbs", "bf16_tflops"):
        if key in peaks:
            assert bench.load_peaks(key) == (float(peaks[key]), "measured")
