"""ClockSampler against a fake nvidia-smi (a shell script on PATH that prints one CSV row
per period), so the sampling logic is tested without a GPU."""
import os
import stat
import time

from opengda_b200.utils.clocks import ClockSampler

FAKE = """#!/bin/bash
i=0
while true; do
  if [ $i -lt 3 ]; then echo "0, 345, 1965, 100.0, 0x0, Not Active, Not Active, Not Active, Not Active";
  else echo "0, 1500, 1965, 990.0, 0x4, Not Active, Not Active, Not Active, Active"; fi
  i=$((i+1)); sleep 0.05
done
"""


def _fake_path(tmp_path, monkeypatch, delay=0.3):
    exe = tmp_path / "nvidia-smi"
    exe.write_text(FAKE.replace("i=0\n", f"sleep {delay}\ni=0\n"))
    exe.chmod(exe.stat().st_mode | stat.S_IEXEC)
    monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ['PATH']}")


def test_sampler_waits_for_first_sample_and_skips_it(tmp_path, monkeypatch):
    _fake_path(tmp_path, monkeypatch)
    with ClockSampler([0]) as cs:
        time.sleep(0.4)  # the "timed region": later rows report 1500 MHz under sw_power_cap
    s = cs.summary()
    assert s["samples"] >= 1
    assert s["sm_max_mhz"] == 1965.0
    assert s["sm_mhz"] >= 345.0
    assert "sw_power_cap" in s["reasons"]


def test_sampler_short_region_still_gets_a_sample(tmp_path, monkeypatch):
    _fake_path(tmp_path, monkeypatch)
    with ClockSampler([0]) as cs:
        pass  # shorter than one period
    assert cs.summary()["samples"] >= 1


def test_sampler_without_nvidia_smi(monkeypatch, tmp_path):
    monkeypatch.setenv("PATH", str(tmp_path))
    with ClockSampler([0]) as cs:
        pass
    assert cs.summary()["reasons"] == ["nvidia-smi unavailable"]
