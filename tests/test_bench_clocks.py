"""The bench's clock record (no GPU): NVML samples decoded into the SM clock and the
active clock-event reasons, against a fake NVML binding."""

import time
from types import SimpleNamespace

import bench


def _fake_nvml(reason_bits):
    """SM clock 1965 MHz; each reasons query returns the next of `reason_bits` (the
    last one repeats)."""
    it = iter(reason_bits)
    last = [reason_bits[-1]]

    def reasons(handle):
        last[0] = next(it, last[0])
        return last[0]

    return SimpleNamespace(
        NVML_CLOCK_SM=1, nvmlDeviceGetClockInfo=lambda h, k: 1965,
        nvmlDeviceGetMaxClockInfo=lambda h, k: 1965,
        nvmlDeviceGetCurrentClocksEventReasons=reasons)


def test_nvml_samples_give_median_clock_and_reason_union(monkeypatch):
    sampler = bench.ClockSampler(0)
    sampler._nvml = object()
    sampler.source = "nvml"
    sampler._bits = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40,
                     "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}
    # 0x1 (GPU idle) is not one of the reasons the record keeps.
    sampler._pynvml = _fake_nvml([0x0, 0x4, 0x4 | 0x1])
    rows = [sampler._sample_nvml() for _ in range(3)]
    assert [r[2] for r in rows] == [frozenset(), {"sw_power_cap"}, {"sw_power_cap"}]
    sampler.rows = rows
    out = sampler.summary()
    assert out["reasons"] == ["sw_power_cap"] and out["samples"] == 3
    assert out["sm_mhz"] == 1965 and out["sm_max_mhz"] == 1965 and out["source"] == "nvml"


def test_sampler_thread_collects_and_stops():
    sampler = bench.ClockSampler(0)
    sampler._nvml = object()
    sampler._bits = {"hw_slowdown": 0x8}
    sampler._pynvml = _fake_nvml([0x8])
    with sampler:
        time.sleep(0.1)
    n = len(sampler.rows)
    assert n >= 2
    time.sleep(0.05)
    assert len(sampler.rows) == n
    assert sampler.summary()["reasons"] == ["hw_slowdown"]
