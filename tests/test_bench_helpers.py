"""bench.py's measurement helpers on the CPU: the algorithmic bytes behind `roofline.achieved`, and
the clock summary behind `clocks` (only samples from the timed region, its throttle reasons)."""
import importlib.util
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def load_bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_algorithmic_bytes_config4():
    b = load_bench()
    # R-MAT 2^24: 263,432,291 entries, 7,379,379 distinct columns, O = 128, fp16 A values and B:
    # A (int32 column + fp16 value), row_ptr, the distinct rows of B, C (fp32) written once
    assert b.algorithmic_bytes(263_432_291, 1 << 24, 7_379_379, 128, 2) == 12_126_758_230
    # fp32 values and B: 8 bytes per entry and 512 bytes per B row
    assert b.algorithmic_bytes(10, 4, 3, 128, 4) == 10 * 8 + 5 * 4 + 3 * 128 * 4 + 4 * 128 * 4


def sample(mhz, max_mhz=1965, power_cap=False, thermal=False):
    flags = ["Not Active"] * 4
    if thermal:
        flags[1] = "Active"
    if power_cap:
        flags[3] = "Active"
    return f"0, {mhz}, {max_mhz}, 900.0, 0x0, " + ", ".join(flags)


def test_clock_summary_keeps_the_timed_region():
    b = load_bench()
    lines = [(0.0, sample(1000)), (0.1, sample(1100)),                 # idle, before the region
             (1.0, sample(1965)), (1.05, sample(1950, power_cap=True)), (1.1, sample(1965)),
             (1.3, sample(900, thermal=True))]                         # after the region
    s = b.summarize_clock_samples(lines, window=(0.95, 1.12))
    assert s["samples"] == 3 and s["timed_region_only"]
    assert s["sm_mhz"] == 1965.0 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"]


def test_clock_summary_falls_back_to_all_samples():
    b = load_bench()
    lines = [(0.0, sample(1965)), (0.5, sample(1965, thermal=True)), (0.6, "garbage"), (0.7, "1, x, y")]
    s = b.summarize_clock_samples(lines, window=(10.0, 10.01))  # no sample inside
    assert s["samples"] == 2 and not s["timed_region_only"]
    assert s["reasons"] == ["hw_thermal_slowdown"]
    none = b.summarize_clock_samples([], window=None)
    assert none["samples"] == 0 and none["sm_mhz"] is None


def test_sampler_without_nvidia_smi():
    b = load_bench()
    c = b.ClockSampler(0)  # never started: as when nvidia-smi is missing
    s = c.stop(window=(0.0, 1.0))
    assert s["samples"] == 0 and s["timed_region_only"] is False and s["reasons"] == ["nvidia-smi unavailable"]
