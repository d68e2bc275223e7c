"""Sanitizer runs of the host side of kiwi::queue and kiwi::invoke (CPU).

Builds tests/native/host_queue_stress.cpp twice, with -fsanitize=thread and
with -fsanitize=address,undefined, and runs each case (SPSC D2H with
wrap-around and back-pressure, MPSC D2H with four CPU stand-ins for the
device producers, SPSC H2D with a CPU stand-in consumer,
concurrent MPMC producers, MPMC producers and CPU stand-in consumers, an invoke Context served by progress threads while
four producers push, the native print formatter from two threads, the host
reader over random ring contents, random callback ids and sizes through the
dispatcher, descriptor exchange between four thread "ranks").  Ring words
are atomic accesses and the writer's release fence is not modelled by TSan
(-Wno-tsan); what TSan checks is every other piece of shared state: cursors,
positions, registries, counters, thread start/stop.  ASan / UBSan check every
buffer and integer operation on those paths.
"""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
CASES = ["spsc_d2h", "mpsc", "spsc_h2d", "mpmc_push", "mpmc", "invoke", "invoke_active", "print", "fuzz", "fuzz_invoke", "fds"]
SANITIZERS = {"thread": ["-fsanitize=thread", "-Wno-tsan"],
              "address,undefined": ["-fsanitize=address,undefined", "-fno-omit-frame-pointer",
                                    "-fno-sanitize-recover=undefined"]}


def _build(tmp_path_factory, name):
    cxx = shutil.which("g++")
    if cxx is None or not os.path.isdir(os.path.join(CUDA, "include")):
        pytest.skip("needs g++ and the CUDA headers")
    out = str(tmp_path_factory.mktemp("san") / ("host_queue_stress_" + name.replace(",", "_")))
    cmd = [cxx, "-std=c++17", "-O1", "-g", *SANITIZERS[name], "-I" + os.path.join(ROOT, "include"),
           "-I" + os.path.join(CUDA, "include"), os.path.join(ROOT, "tests/native/host_queue_stress.cpp"),
           os.path.join(ROOT, "src/queue/host_memory.cpp"), os.path.join(ROOT, "src/common/topology.cpp"),
           os.path.join(ROOT, "src/p2p/fd_exchange.cpp"),
           "-L" + os.path.join(CUDA, "lib64"), "-lcudart", "-lpthread", "-o", out]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    if r.returncode != 0 and "cannot find" in r.stderr.lower() and "san" in r.stderr.lower():
        pytest.skip("no sanitizer runtime: " + r.stderr.strip().splitlines()[-1])
    assert r.returncode == 0, r.stderr[-4000:]
    return out


@pytest.fixture(scope="module", params=sorted(SANITIZERS))
def binary(request, tmp_path_factory):
    return request.param, _build(tmp_path_factory, request.param)


@pytest.mark.parametrize("case", CASES)
def test_host_queues_under_sanitizers(binary, case):
    name, path = binary
    env = dict(os.environ, TSAN_OPTIONS="halt_on_error=1 exitcode=66",
               ASAN_OPTIONS="detect_leaks=1:halt_on_error=1:exitcode=66", UBSAN_OPTIONS="halt_on_error=1",
               LD_LIBRARY_PATH=os.path.join(CUDA, "lib64") + ":" + os.environ.get("LD_LIBRARY_PATH", ""))
    r = subprocess.run([path, case], capture_output=True, text=True, timeout=240, env=env)
    out = r.stdout + r.stderr
    for marker in ("ThreadSanitizer", "AddressSanitizer", "LeakSanitizer", "runtime error:"):
        assert marker not in out, f"[{name}] " + out[-6000:]
    assert r.returncode == 0, f"[{name}] " + out[-4000:]
    assert f"{case} ok" in r.stdout
