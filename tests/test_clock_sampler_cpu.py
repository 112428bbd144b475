"""The bench's multi-rank clock sampler (an ``nvidia-smi -lms`` process) against a fake
nvidia-smi on CPU: samples around the timed region are kept, reasons decoded, the process
ended."""
import os
import stat
import sys
import time
import types

import bench


def _fake_smi(tmp_path, reasons="0x0000000000000004"):
    script = tmp_path / "nvidia-smi"
    script.write_text(f"""#!{sys.executable}
import datetime, sys, time
for _ in range(400):   # bounded: 8 s at most
    now = datetime.datetime.now().strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
    print(f"{{now}}, 1965, 1965, 612.25, {reasons}", flush=True)
    time.sleep(0.02)
""")
    script.chmod(script.stat().st_mode | stat.S_IEXEC)
    return tmp_path


def test_smi_sampler_keeps_samples_around_the_region(tmp_path, monkeypatch):
    monkeypatch.setenv("PATH", f"{_fake_smi(tmp_path)}{os.pathsep}{os.environ['PATH']}")
    props = types.SimpleNamespace(pci_domain_id=0, pci_bus_id=0x1B, pci_device_id=0)
    monkeypatch.setattr(bench.torch.cuda, "get_device_properties", lambda index: props)
    monkeypatch.setenv("WORLD_SIZE", "2")
    sampler = bench.ClockSampler(0)
    assert isinstance(sampler, bench._SmiClockSampler) and sampler.ok
    sampler.start()
    time.sleep(0.1)
    clocks = sampler.stop()
    assert clocks["source"] == "nvidia-smi"
    assert clocks["samples"] >= 2
    assert clocks["sm_mhz"] == 1965 and clocks["sm_max_mhz"] == 1965
    assert clocks["reasons"] == ["sw_power_cap"] and clocks["power_w_max"] == 612.25
    assert sampler.proc.poll() is not None


def test_single_rank_uses_nvml_sampler(monkeypatch):
    monkeypatch.setenv("WORLD_SIZE", "1")
    sampler = bench.ClockSampler(0)
    assert isinstance(sampler, bench._NvmlClockSampler)
