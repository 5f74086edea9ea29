"""Host-side pieces of bench.py (no GPU): throttle-reason decoding of the clock samples
and the JSON fields they feed."""
import bench


def test_nvml_samples_decode_reasons_and_median():
    c = bench.ClockSampler.__new__(bench.ClockSampler)
    c.samples, c.lines, c.max_mhz = [(1965.0, 0), (1800.0, 0x4), (1965.0, 0x40), (1900.0, 0x8 | 0x20)], [], 1965.0
    s = c.summary()
    assert s["source"] == "nvml" and s["samples"] == 4
    assert s["sm_mhz"] == 1932.5 and s["sm_min_mhz"] == 1800.0 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["hw_slowdown", "hw_thermal_slowdown", "sw_power_cap", "sw_thermal_slowdown"]


def test_nvidia_smi_lines_are_the_fallback():
    c = bench.ClockSampler.__new__(bench.ClockSampler)
    c.samples = []
    c.lines = ["0, 1965, 1965, 700.5, 0x0, Not Active, Not Active, Not Active, Not Active",
               "0, 1400, 1965, 990.1, 0x4, Not Active, Not Active, Not Active, Active",
               "garbled"]
    s = c.summary()
    assert s["source"] == "nvidia-smi" and s["samples"] == 2
    assert s["sm_mhz"] == 1682.5 and s["reasons"] == ["sw_power_cap"]


def test_no_samples_reports_none():
    c = bench.ClockSampler.__new__(bench.ClockSampler)
    c.samples, c.lines = [], []
    assert c.summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}


def test_peaks_come_from_the_measured_file_or_the_fallback():
    burst, sustained, hbm, src = bench.measured_peaks()
    assert src in ("measured", "fallback") and burst >= sustained > 0 and hbm > 0
