"""Clock sampling (CPU): a stand-in ``nvidia-smi`` on PATH prints the CSV fields the
sampler asks for; the summary gives the median SM clock under load, the max clock and
the throttle reasons that were active."""
import os
import stat
import time

from spec_ep.utils.clocks import ClockSampler

FAKE = """#!/bin/sh
echo "$@" > "{args}"
printf '0, 1800, 1965, 900.1, 0x4, Not Active, Not Active, Not Active, Active\\n'
printf '0, 1900, 1965, 950.0, 0x0, Not Active, Not Active, Not Active, Not Active\\n'
printf '0, 1850, 1965, 990.5, 0x4, Not Active, Not Active, Not Active, Active\\n'
printf 'garbage line\\n'
sleep 30
"""


def test_sampler_summarises_a_stand_in_nvidia_smi(tmp_path, monkeypatch):
    args = tmp_path / "args.txt"
    exe = tmp_path / "nvidia-smi"
    exe.write_text(FAKE.format(args=args))
    exe.chmod(exe.stat().st_mode | stat.S_IXUSR)
    monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ['PATH']}")
    with ClockSampler("GPU-1234", period_ms=100) as clk:
        for _ in range(100):  # until the stand-in has printed its lines
            if args.exists() and os.path.getsize(clk.path) > 200:
                break
            time.sleep(0.05)
    s = clk.summary()
    assert s == {"sm_mhz": 1850.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 3}
    called = args.read_text()
    assert "--id=GPU-1234" in called and "-lms=100" in called and "clocks_event_reasons.sw_power_cap" in called


def test_sampler_without_nvidia_smi_reports_unsampled(tmp_path, monkeypatch):
    monkeypatch.setenv("PATH", str(tmp_path))  # no nvidia-smi anywhere
    with ClockSampler(None) as clk:
        pass
    assert clk.summary()["reasons"] == ["unsampled"]
