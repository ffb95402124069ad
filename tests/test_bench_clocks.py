"""bench.py's clock sampler (the SM clock and throttle reasons recorded beside
every bench line), on the CPU against a stand-in nvidia-smi that prints one
CSV sample every 200 ms:
  * a timed region shorter than the sampling interval still gets the sample
    that closes it;
  * a longer region gets the samples taken inside it, not those before it;
  * a throttle reason reported active appears in the summary;
  * a local GPU index is mapped through CUDA_VISIBLE_DEVICES;
  * without nvidia-smi the summary says "unsampled" instead of failing."""
import os
import stat
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def fake_smi(tmp_path, line):
    exe = tmp_path / "nvidia-smi"
    exe.write_text("#!/bin/bash\n"
                   f"echo \"$@\" > {tmp_path / 'args'}\n"
                   "sleep 0.1\n"
                   f"while true; do echo '{line}'; sleep 0.2; done\n")
    exe.chmod(exe.stat().st_mode | stat.S_IEXEC)
    return exe


def with_path(tmp_path, monkeypatch, cvd=None):
    monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ.get('PATH', '')}")
    if cvd is None:
        monkeypatch.delenv("CUDA_VISIBLE_DEVICES", raising=False)
    else:
        monkeypatch.setenv("CUDA_VISIBLE_DEVICES", cvd)


def test_short_region_gets_one_sample(tmp_path, monkeypatch):
    fake_smi(tmp_path, "0, 1965, 1965, 400.0, 0x0, Not Active, Not Active, Not Active, Not Active")
    with_path(tmp_path, monkeypatch)
    c = bench.ClockSampler(0)
    with c:
        time.sleep(0.02)
    s = c.summary()
    assert s["samples"] >= 1 and s["sm_mhz"] == 1965.0 and s["reasons"] == []


def test_long_region_and_reasons(tmp_path, monkeypatch):
    fake_smi(tmp_path, "0, 1300, 1965, 1000.0, 0x4, Not Active, Not Active, Not Active, Active")
    with_path(tmp_path, monkeypatch)
    c = bench.ClockSampler(0)
    with c:
        time.sleep(0.7)
    s = c.summary()
    assert 2 <= s["samples"] <= 6
    assert s["sm_mhz"] == 1300.0 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"]


def test_visible_devices_mapping(tmp_path, monkeypatch):
    fake_smi(tmp_path, "5, 1965, 1965, 400.0, 0x0, Not Active, Not Active, Not Active, Not Active")
    with_path(tmp_path, monkeypatch, cvd="3,5")
    c = bench.ClockSampler(1)
    assert c.gpu == "5"
    with c:
        time.sleep(0.02)
    assert "-i 5" in (tmp_path / "args").read_text()


def test_without_nvidia_smi(tmp_path, monkeypatch):
    monkeypatch.setenv("PATH", str(tmp_path))   # an empty directory
    c = bench.ClockSampler(0)
    with c:
        pass
    assert c.summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
