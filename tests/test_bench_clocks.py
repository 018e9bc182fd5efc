"""bench.py's clock record, from samples given directly (no GPU, no NVML): the
median SM clock, the throttle reasons that were active at any sample (the
ones that reject a measurement: hw_slowdown, hw_thermal_slowdown,
sw_thermal_slowdown; sw_power_cap is kept and noted), and the flag on a
record of fewer than 10 samples. Both sources: NVML reason bits and
nvidia-smi's CSV."""
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402


def nvml_sampler(samples, max_mhz=1965):
    s = bench.ClockSampler(0)
    s.thread = object()  # summary() reads the NVML samples when a poller ran
    s.samples = list(samples)
    s.max_mhz = max_mhz
    return s


def test_nvml_median_and_no_reasons():
    out = nvml_sampler([(1965, 0)] * 9 + [(1950, 0)] * 4).summary()
    assert out["sm_mhz"] == 1965.0 and out["sm_max_mhz"] == 1965.0
    assert out["reasons"] == [] and out["samples"] == 13 and "note" not in out


def test_nvml_reason_bits():
    # idle (0x1) and sync boost (0x10) are not reasons that matter here
    out = nvml_sampler([(1965, 0x1), (1800, 0x4), (1700, 0x4 | 0x8), (1600, 0x20), (1500, 0x40 | 0x10)] * 2).summary()
    assert out["reasons"] == ["hw_slowdown", "hw_thermal_slowdown", "sw_power_cap", "sw_thermal_slowdown"]
    assert out["sm_mhz"] == 1700.0


def test_few_samples_are_flagged():
    out = nvml_sampler([(1965, 0)] * 3).summary()
    assert out["samples"] == 3 and "unreliable" in out["note"]
    assert nvml_sampler([]).summary()["reasons"] == ["unsampled"]


def test_nvidia_smi_csv(tmp_path):
    rows = [
        "0, 1965, 1965, 700.1, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
        "0, 1900, 1965, 998.0, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "0, 1965, 1965, 990.5, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "garbage line",
    ]
    p = tmp_path / "clocks.csv"
    p.write_text("\n".join(rows) + "\n")
    s = bench.ClockSampler(0)
    s.path = str(p)
    out = s.summary()
    assert out["source"] == "nvidia-smi" and out["samples"] == 3
    assert out["sm_mhz"] == 1965.0 and out["sm_max_mhz"] == 1965.0
    assert out["reasons"] == ["sw_power_cap"]
    p.write_text("0, 1400, 1965, 500, 0x48, Active, Active, Not Active, Not Active\n")
    assert bench.ClockSampler.summary(s)["reasons"] == ["hw_slowdown", "hw_thermal_slowdown"]
