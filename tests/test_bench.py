"""Host-side pieces of bench.py (no GPU): the clock summary the JSON line carries.

The timing rules reject a run that saw hw_slowdown, hw_thermal_slowdown or sw_thermal_slowdown, and note sw_power_cap;
the summary must report every reason seen in any sample (NVML bit masks or nvidia-smi rows) and the median SM clock.
"""
import importlib.util
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("d1_bench", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_clock_summary_nvml(bench):
    c = bench.Clocks(0)
    c.max_mhz = 1965.0
    c.samples = [(1965.0, 0), (1950.0, 0x4), (1965.0, 0), (1500.0, 0x8 | 0x40)]
    s = c.summary()
    assert s["sm_mhz"] == 1957.5 and s["sm_max_mhz"] == 1965.0 and s["samples"] == 4 and s["source"] == "nvml"
    assert s["reasons"] == ["hw_slowdown", "hw_thermal_slowdown", "sw_power_cap"]


def test_clock_summary_nvidia_smi(bench):
    c = bench.Clocks(0)
    c.lines = ["0, 1965, 1965, 800.1, 0x0, Not Active, Not Active, Not Active, Not Active",
               "0, 1800, 1965, 990.0, 0x4, Not Active, Not Active, Active, Active",
               "garbage"]
    s = c.summary()
    assert s["sm_mhz"] == 1882.5 and s["sm_max_mhz"] == 1965.0 and s["samples"] == 2 and s["source"] == "nvidia-smi"
    assert s["reasons"] == ["sw_power_cap", "sw_thermal_slowdown"]


def test_clock_summary_unsampled(bench):
    assert bench.Clocks(0).summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
