"""The bench.py contract on CPU: the reference arm's JSON line, the kernel
count per step, and the clock sampler that bench.py runs during the timed
region (driven here by a stand-in nvidia-smi that prints fixed samples)."""
import json
import os
import stat
import subprocess
import sys
import time

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_unavailable_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference"], capture_output=True,
                       text=True, timeout=300, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unavailable"]


def test_kernels_per_step_counts_each_path():
    sys.path.insert(0, ROOT)
    import bench

    assert bench.kernels_per_step(True, False) == 13
    assert bench.kernels_per_step(False, False) == 14
    assert bench.kernels_per_step(True, True) == 12


@pytest.fixture()
def fake_smi(tmp_path, monkeypatch):
    script = tmp_path / "nvidia-smi"
    # index, sm, max, power, hw_slowdown, hw_thermal, sw_thermal, sw_power_cap
    script.write_text("#!/bin/sh\n"
                      "i=0\n"
                      "while [ $i -lt 40 ]; do\n"
                      "  if [ $i -ge 10 ] && [ $i -lt 20 ]; then\n"
                      "    echo '0, 1800, 1965, 950.5, Not Active, Not Active, Not Active, Active'\n"
                      "  else\n"
                      "    echo '0, 1965, 1965, [N/A], Not Active, Not Active, Not Active, Not Active'\n"
                      "  fi\n"
                      "  i=$((i+1)); sleep 0.02\n"
                      "done\n")
    script.chmod(script.stat().st_mode | stat.S_IEXEC)
    monkeypatch.setenv("PATH", str(tmp_path) + os.pathsep + os.environ["PATH"])
    return script


def test_clock_sampler_summarises_the_timed_region(fake_smi):
    from kiwi_b200.utils.clocks import ClockSampler

    cs = ClockSampler(device_index=0, period_ms=20)
    with cs:
        cs.wait_first_sample()
        cs.mark_start()
        time.sleep(0.5)
        cs.mark_end()
    s = cs.summary()
    assert s["samples"] > 5
    assert s["sm_max_mhz"] == 1965
    assert 1800 <= s["sm_mhz"] <= 1965
    assert s["reasons"] in ([], ["sw_power_cap"])
    all_reasons = set().union(*(x[4] for x in cs.samples))
    assert all_reasons == {"sw_power_cap"}  # parsed from the 'Active' column
    assert any(x[3] is None for x in cs.samples) and any(x[3] == 950.5 for x in cs.samples)


def test_clock_sampler_without_nvidia_smi(monkeypatch, tmp_path):
    from kiwi_b200.utils.clocks import ClockSampler

    monkeypatch.setenv("PATH", str(tmp_path))
    with ClockSampler() as cs:
        cs.wait_first_sample(timeout_s=0.1)
        cs.mark_start()
        cs.mark_end()
    assert cs.summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
