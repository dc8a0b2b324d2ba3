"""The bench line's clock record: nvidia-smi lines and NVML samples merge into one median and one set of
active throttle reasons (no GPU: the samples are injected)."""
import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_for_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_clock_summary_merges_both_sources():
    pynvml = pytest.importorskip("pynvml")
    c = _bench().ClockSampler(0)
    c.lines = ["0, 1965, 1965, 700.1, 0x0, Not Active, Not Active, Not Active, Not Active",
               "0, 1950, 1965, 980.0, 0x4, Not Active, Not Active, Not Active, Active"]
    c.nvml = [(1965.0, 0), (1965.0, 0), (1900.0, int(pynvml.nvmlClocksEventReasonHwSlowdown))]
    s = c.summary()
    assert s["samples"] == 5 and s["samples_nvidia_smi"] == 2 and s["samples_nvml"] == 3
    assert s["sm_mhz"] == 1965.0 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["hw_slowdown", "sw_power_cap"]


def test_clock_summary_nvml_only_takes_the_nvml_maximum():
    pytest.importorskip("pynvml")
    c = _bench().ClockSampler(0)
    c.nvml = [(1327.0, 0)]
    c.nvml_max = 1965.0
    s = c.summary()
    assert s["sm_mhz"] == 1327.0 and s["sm_max_mhz"] == 1965.0 and s["reasons"] == []


def test_clock_sampler_without_a_gpu_records_nothing():
    c = _bench().ClockSampler(0)
    with c:
        pass
    assert c.summary()["samples"] == len(c.nvml) + c.summary()["samples_nvidia_smi"]
