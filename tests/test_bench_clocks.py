"""bench.py's clock record: nvidia-smi samples taken inside the timed region only.

A stand-in `nvidia-smi` on PATH prints timestamped rows in the format the
sampler asks for, so the parsing, the in-region filter and the throttle
reasons are checked without a GPU."""
import os
import stat
import sys
import time

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
import bench  # noqa: E402

FAKE = """#!{python}
import datetime, sys, time
while True:
    now = datetime.datetime.now().strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
    print(f"{{now}}, 0, {sm}, 1965, 640.5, 0x0000000000000004, {hw}, Not Active, Not Active, {cap}", flush=True)
    time.sleep(0.02)
"""


def _fake_smi(tmp_path, monkeypatch, sm=1410, hw="Not Active", cap="Active"):
    d = tmp_path / "bin"
    d.mkdir()
    p = d / "nvidia-smi"
    p.write_text(FAKE.format(python=sys.executable, sm=sm, hw=hw, cap=cap))
    p.chmod(p.stat().st_mode | stat.S_IEXEC)
    monkeypatch.setenv("PATH", f"{d}{os.pathsep}{os.environ['PATH']}")


def test_samples_inside_the_region_with_power_cap(tmp_path, monkeypatch):
    _fake_smi(tmp_path, monkeypatch)
    c = bench.ClockSampler(0)
    c.begin()
    time.sleep(0.3)
    rec = c.stop()
    assert rec["samples_in_region"] >= 5
    assert rec["sm_mhz"] == 1410.0 and rec["sm_max_mhz"] == 1965.0
    assert rec["reasons"] == ["sw_power_cap"]
    assert rec["power_w_max"] == pytest.approx(640.5)


def test_hardware_slowdown_is_reported(tmp_path, monkeypatch):
    _fake_smi(tmp_path, monkeypatch, sm=900, hw="Active", cap="Not Active")
    c = bench.ClockSampler(0)
    c.begin()
    time.sleep(0.15)
    rec = c.stop()
    assert rec["reasons"] == ["hw_slowdown"] and rec["sm_mhz"] == 900.0


def test_region_shorter_than_a_sample_takes_the_nearest(tmp_path, monkeypatch):
    _fake_smi(tmp_path, monkeypatch)
    c = bench.ClockSampler(0)
    time.sleep(0.1)
    c.begin()
    rec = c.stop()  # no sample can fall inside a region this short
    assert rec["samples_in_region"] in (0, 1) and rec["sm_mhz"] == 1410.0


def test_no_nvidia_smi_gives_no_record(tmp_path, monkeypatch):
    empty = tmp_path / "empty"
    empty.mkdir()
    monkeypatch.setenv("PATH", str(empty))
    c = bench.ClockSampler(0)
    c.begin()
    assert c.stop() is None


class FakeNvml:
    """Stand-in for pynvml: fixed SM clock, power and clock-event reason bits."""
    NVML_CLOCK_SM = 1

    def __init__(self, sm=1350, bits=0x4):
        self.sm, self.bits = sm, bits

    def nvmlInit(self):
        pass

    def nvmlDeviceGetHandleByUUID(self, uuid):
        raise RuntimeError("no uuid lookup here")

    def nvmlDeviceGetHandleByIndex(self, i):
        return ("gpu", i)

    def nvmlDeviceGetMaxClockInfo(self, h, which):
        return 1965

    def nvmlDeviceGetClockInfo(self, h, which):
        return self.sm

    def nvmlDeviceGetPowerUsage(self, h):
        return 990500  # mW

    def nvmlDeviceGetCurrentClocksEventReasons(self, h):
        return self.bits


def test_nvml_sampler_polls_inside_the_region():
    c = bench.NvmlClockSampler(0, nvml=FakeNvml())
    time.sleep(0.05)
    c.begin()
    time.sleep(0.2)
    rec = c.stop()
    assert rec["source"] == "nvml" and rec["period_ms"] == 10
    assert rec["samples_in_region"] >= 8  # a 10 ms period lands many samples in a 30 ms region and more
    assert rec["sm_mhz"] == 1350.0 and rec["sm_max_mhz"] == 1965.0
    assert rec["reasons"] == ["sw_power_cap"] and rec["power_w_max"] == pytest.approx(990.5)


def test_nvml_sampler_reports_thermal_and_hw_slowdown():
    c = bench.NvmlClockSampler(0, nvml=FakeNvml(sm=700, bits=0x8 | 0x40))
    c.begin()
    time.sleep(0.05)
    rec = c.stop()
    assert rec["reasons"] == ["hw_slowdown", "hw_thermal_slowdown"] and rec["sm_mhz"] == 700.0
