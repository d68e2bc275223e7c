"""The CMake build for C++ applications: configure, build and install the
kiwi libraries (sm_100a objects, cross-compiled without a GPU), then build a
separate project that finds them with find_package(kiwi) and links kiwi::ep and
kiwi::invoke, and run it (host-only calls)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(cmd, cwd):
    r = subprocess.run(cmd, cwd=cwd, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, f"{' '.join(cmd)}\n{r.stdout[-3000:]}\n{r.stderr[-3000:]}"
    return r.stdout


@pytest.mark.skipif(shutil.which("cmake") is None or shutil.which("nvcc") is None and
                    not os.path.exists("/usr/local/cuda/bin/nvcc"), reason="needs cmake and nvcc")
def test_cmake_build_install_and_find_package(tmp_path):
    env_gen = ["-G", "Ninja"] if shutil.which("ninja") else []
    build, prefix, consumer = tmp_path / "b", tmp_path / "prefix", tmp_path / "c"
    _run(["cmake", "-S", ROOT, "-B", str(build), *env_gen, "-DKIWI_BUILD_EXAMPLES=OFF", "-DKIWI_BUILD_BENCH=OFF"],
         ROOT)
    _run(["cmake", "--build", str(build), "-j", str(min(8, os.cpu_count() or 1))], ROOT)
    _run(["cmake", "--install", str(build), "--prefix", str(prefix)], ROOT)
    for lib in ("queue", "topology", "p2p", "gemm", "ops", "ep"):
        assert any(p.name == f"libkiwi_{lib}.a" for p in prefix.rglob("*.a")), lib
    assert (prefix / "include" / "kiwi" / "gemm" / "noalloc.h").exists()
    _run(["cmake", "-S", os.path.join(ROOT, "tests", "cmake_consumer"), "-B", str(consumer), *env_gen,
          f"-DCMAKE_PREFIX_PATH={prefix}"], ROOT)
    _run(["cmake", "--build", str(consumer)], ROOT)
    out = _run([str(consumer / "kiwi_consumer")], ROOT)
    fields = dict(kv.split("=") for kv in out.split())
    assert fields["experts_per_rank"] == "32" and int(fields["heap_bytes"]) > 0
    assert fields["recv_blocks"] == str(8 * 148) and fields["m64"] == "1"
    assert fields["max_groups"] == "1024" and fields["cpus"] == "5"
