"""Host logic of bench.py that the driver relies on, on the CPU.

* ClockSampler keeps only the nvidia-smi samples taken inside the timed region and
  reports throttle reasons from them (a fake nvidia-smi stands in for the real one).
* emit() writes exactly one JSON line per result to the original stdout, whatever
  else the process prints (run as a child process so its fd juggling stays there).
"""
import json
import os
import stat
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _fake_smi(tmp_path, line):
    exe = tmp_path / "nvidia-smi"
    exe.write_text("#!/bin/bash\nwhile true; do echo '%s'; sleep 0.01; done\n" % line)
    exe.chmod(exe.stat().st_mode | stat.S_IEXEC)
    return str(tmp_path)


def test_clock_sampler_window_and_reasons(tmp_path, monkeypatch):
    import bench
    d = _fake_smi(tmp_path, "0, 1900, 1965, 900.5, 0x4, Not Active, Not Active, Not Active, Active")
    monkeypatch.setenv("PATH", d + os.pathsep + os.environ["PATH"])
    with bench.ClockSampler(0) as clk:
        time.sleep(0.15)
    time.sleep(0.1)  # samples after the region must not count
    s = clk.summary()
    assert s["samples"] >= 1
    assert s["sm_mhz"] == 1900.0 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"]
    inside = [t for t, _ in clk.rows if clk.t_start <= t <= clk.t_end + 0.025]
    assert len(inside) == s["samples"] <= len(clk.rows)


def test_clock_sampler_without_nvidia_smi(tmp_path, monkeypatch):
    import bench
    monkeypatch.setenv("PATH", str(tmp_path))  # no nvidia-smi anywhere
    with bench.ClockSampler(0) as clk:
        pass
    assert clk.summary()["reasons"] == ["unavailable"]


def test_emit_keeps_stdout_to_result_lines():
    code = (
        "import os, sys; sys.path.insert(0, %r); import bench\n"
        "bench._OUT_FD = os.dup(1); os.dup2(2, 1)\n"
        "print('noise from python'); os.write(1, b'noise from C\\n')\n"
        "bench.emit({'metric': 'm', 'value': 1.5})\n" % REPO)
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    lines = out.stdout.strip().splitlines()
    assert len(lines) == 1 and json.loads(lines[0]) == {"metric": "m", "value": 1.5}
    assert "noise from python" in out.stderr and "noise from C" in out.stderr
