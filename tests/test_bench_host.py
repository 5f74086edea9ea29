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


def test_whole_path_workloads_have_the_configured_shapes():
    """P_lin of the workload models equals the configurations' (GPT-2 small / medium / XL, Qwen3-style)."""
    from opus_b200.layers import GCLinear
    from opus_b200.train import data_selection as ds

    want = {"gpt2-small": 84_934_656, "gpt2-medium": 301_989_888, "gpt2-xl": 1_474_560_000,
            "qwen3": 1_409_286_144}
    for name, p_lin in want.items():
        cfg = dict(bench.WHOLE[name])
        assert bench.capture_layer_weights(cfg) == p_lin, name
        one = bench.build_model(cfg, GCLinear, 1)  # one block: the formula per block matches the layers
        layers = ds.find_GClayers(one)
        assert sum(layer.weight.numel() for layer in layers) * cfg["layers"] == p_lin, name
    assert bench.WHOLE["gpt2-xl"]["cand"] * 8 == 1024 and bench.WHOLE["gpt2-xl"]["proxy"] * 8 == 128


def test_zipf_tokens_and_kept_share():
    import numpy as np

    t = bench.zipf_tokens(np.random.default_rng(0), 3, 64, 50257)
    assert t.shape == (3, 64) and t.dtype == np.int64 and t.min() >= 0 and t.max() < 50257
    assert (t == 0).mean() > 0.05  # rank 1 is the most frequent id

    class A:
        workload, candidates, proxies, model_dtype = "gpt2-xl", None, None, None

    cfg = bench.whole_config(A)
    assert cfg["kept"] == 32 and cfg["dtype"] == "bf16"
    A.candidates, A.proxies, A.model_dtype = 16, 0, "f32"
    cfg = bench.whole_config(A)
    assert (cfg["cand"], cfg["proxy"], cfg["kept"], cfg["dtype"]) == (16, 0, 4, "f32")
