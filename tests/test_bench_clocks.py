"""The benchmark's clock record on CPU: the NVML sampling thread (against a
fake NVML module) reports the median loaded SM clock, the maximum and every
clock-event reason seen; the CUDA ordinal is mapped to the physical index
through CUDA_VISIBLE_DEVICES; with neither NVML nor nvidia-smi available the
record is absent rather than invented."""
import threading
import time
import types

import bench


def _fake_nvml(clocks, reasons):
    seq = iter(clocks)
    last = [clocks[-1]]

    def clock(h, kind):
        try:
            last[0] = next(seq)
        except StopIteration:
            pass
        return last[0]

    return types.SimpleNamespace(
        nvmlClocksEventReasonHwSlowdown=0x8, nvmlClocksEventReasonHwThermalSlowdown=0x40,
        nvmlClocksEventReasonSwThermalSlowdown=0x20, nvmlClocksEventReasonSwPowerCap=0x4,
        NVML_CLOCK_SM=1, nvmlDeviceGetMaxClockInfo=lambda h, k: 1965,
        nvmlDeviceGetClockInfo=clock, nvmlDeviceGetCurrentClocksEventReasons=lambda h: reasons)


def _sample(nv, seconds=0.08):
    c = bench.ClockSampler(0)
    c._nv, c._h = nv, None
    c._stop = threading.Event()
    c.thread = threading.Thread(target=c._nvml_loop, args=(nv, None, c._stop))
    c.thread.start()
    time.sleep(seconds)
    return c.stop()


def test_nvml_samples_give_median_max_and_reasons():
    rec = _sample(_fake_nvml([1965, 1965, 1950, 1965, 1965, 1965, 1965, 1965], 0x4 | 0x8))
    assert rec["samples"] >= 3
    assert rec["sm_max_mhz"] == 1965
    assert rec["sm_mhz"] == 1965
    assert rec["reasons"] == ["hw_slowdown", "sw_power_cap"]
    assert "NVML" in rec["source"]


def test_idle_samples_are_left_out_of_the_median():
    # Samples below half the maximum (the GPU idle between steps) do not count.
    rec = _sample(_fake_nvml([345, 1900, 1900, 1900, 1900, 1900, 1900, 1900], 0))
    assert rec["sm_mhz"] == 1900
    assert rec["reasons"] == []


def test_ordinal_maps_through_cuda_visible_devices(monkeypatch):
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "5,3")
    assert bench.ClockSampler(1).index == 3
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "GPU-1234")
    assert bench.ClockSampler(0).index == 0
    monkeypatch.delenv("CUDA_VISIBLE_DEVICES")
    assert bench.ClockSampler(2).index == 2


def test_region_end_is_sampled_even_if_the_thread_took_none():
    # The sample taken by stop() itself: a region shorter than the thread's
    # first poll still gets a record.
    nv = _fake_nvml([1965], 0x4)
    c = bench.ClockSampler(0)
    c._nv, c._h = nv, None
    c._stop = threading.Event()
    c.thread = threading.Thread(target=lambda: None)
    c.thread.start()
    rec = c.stop()
    assert rec["samples"] == 1 and rec["sm_mhz"] == 1965 and rec["reasons"] == ["sw_power_cap"]


def test_no_sources_give_no_record():
    c = bench.ClockSampler(0)
    assert c.stop() is None
