"""CPU checks of bench.py's host side: the clock sampler (against a fake
nvidia-smi on PATH) and the reference arm's JSON line on configuration 1."""

import json
import os
import subprocess
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
FAKE = """#!/bin/bash
sleep 0.3
while true; do echo "0, {mhz}, 1965, 900.0, 0x4, {hw}, Not Active, Not Active, Active"; sleep 0.05; done
"""


def fake_smi(tmp_path, monkeypatch, mhz, hw):
    exe = tmp_path / "nvidia-smi"
    exe.write_text(FAKE.format(mhz=mhz, hw=hw))
    exe.chmod(0o755)
    monkeypatch.setenv("PATH", f"{tmp_path}:{os.environ['PATH']}")


def test_clock_sampler_samples_a_short_region_after_a_slow_start(tmp_path, monkeypatch):
    """nvidia-smi's first sample arrives 0.3 s after launch; a 0.12 s region is still sampled."""
    fake_smi(tmp_path, monkeypatch, 1900, "Not Active")
    sys.path.insert(0, str(REPO))
    import bench

    with bench.ClockSampler(0) as clocks:
        time.sleep(0.12)
    got = clocks.summary()
    assert got["samples"] >= 1 and got["sm_mhz"] == 1900.0 and got["sm_max_mhz"] == 1965.0
    assert got["reasons"] == ["sw_power_cap"]


def test_clock_sampler_reports_hardware_slowdown(tmp_path, monkeypatch):
    fake_smi(tmp_path, monkeypatch, 1100, "Active")
    sys.path.insert(0, str(REPO))
    import bench

    with bench.ClockSampler(0) as clocks:
        time.sleep(0.12)
    assert "hw_slowdown" in clocks.summary()["reasons"]


def test_reference_arm_prints_the_contract_line():
    """`bench.py --impl reference` runs the float64 CPU restatement on a bounded sample and
    prints one JSON line with the reference arm's keys."""
    res = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--config", "1", "--steps", "1",
                          "--warmup", "0", "--cpu-sample-tokens", "8"], capture_output=True, text=True, timeout=300,
                         cwd=REPO)
    assert res.returncode == 0, res.stderr[-2000:]
    line = json.loads(res.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0 and line["unit"] == "tokens/s"
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["higher_is_better"] is True and line["config"]["workload"].startswith("cfg1")
