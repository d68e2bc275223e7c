"""ThreadSanitizer run of the host side of kiwi::queue and kiwi::invoke (CPU).

Builds tests/native/tsan_host_queues.cpp with -fsanitize=thread and runs each
case (SPSC D2H with wrap-around and back-pressure, SPSC H2D with a CPU stand-in
consumer, concurrent MPMC producers, an invoke Context served by progress
threads while four producers push).  Ring words are atomic accesses and the
writer's release fence is not modelled by TSan (-Wno-tsan); what TSan checks is
every other piece of shared state: cursors, positions, registries, counters,
thread start/stop.
"""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
CASES = ["spsc_d2h", "spsc_h2d", "mpmc_push", "invoke"]


@pytest.fixture(scope="module")
def binary(tmp_path_factory):
    cxx = shutil.which("g++")
    if cxx is None or not os.path.isdir(os.path.join(CUDA, "include")):
        pytest.skip("needs g++ and the CUDA headers")
    out = str(tmp_path_factory.mktemp("tsan") / "tsan_host_queues")
    cmd = [cxx, "-std=c++17", "-O1", "-g", "-fsanitize=thread", "-Wno-tsan", "-I" + os.path.join(ROOT, "include"),
           "-I" + os.path.join(CUDA, "include"), os.path.join(ROOT, "tests/native/tsan_host_queues.cpp"),
           os.path.join(ROOT, "src/queue/host_memory.cpp"), os.path.join(ROOT, "src/common/topology.cpp"),
           "-L" + os.path.join(CUDA, "lib64"), "-lcudart", "-lpthread", "-o", out]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    if r.returncode != 0 and ("tsan" in r.stderr.lower() and "cannot find" in r.stderr.lower()):
        pytest.skip("no ThreadSanitizer runtime: " + r.stderr.strip().splitlines()[-1])
    assert r.returncode == 0, r.stderr[-4000:]
    return out


@pytest.mark.parametrize("case", CASES)
def test_host_queues_are_race_free(binary, case):
    env = dict(os.environ, TSAN_OPTIONS="halt_on_error=1 exitcode=66",
               LD_LIBRARY_PATH=os.path.join(CUDA, "lib64") + ":" + os.environ.get("LD_LIBRARY_PATH", ""))
    r = subprocess.run([binary, case], capture_output=True, text=True, timeout=240, env=env)
    out = r.stdout + r.stderr
    assert "ThreadSanitizer" not in out, out[-6000:]
    assert r.returncode == 0, out[-4000:]
    assert f"{case} ok" in r.stdout
