"""Build helpers for user CUDA code that uses the kiwi headers.

``load_inline(name, cuda_sources, functions)`` wraps
``torch.utils.cpp_extension.load_inline`` with the repository's ``include/``
directory and sm_100a code generation, so a user kernel can
``#include <kiwi/invoke/device_context.cuh>`` and call host callbacks that a
:class:`kiwi_b200.invoke.Context` registered (pass ``ctx.device_context_ptr``
to the kernel as a ``kiwi::invoke::DeviceContext<kiwi::queue::SPSCD2HQueue>*``).
This is the PyTorch-level replacement of the reference's Triton / FlyDSL
frontends (python/kiwi_triton.py, python/kiwi_flydsl of AMDResearch/kiwi).

``load_cuda(name, cuda_source)`` is the light-weight alternative: nvcc alone
builds the source (kiwi headers, no PyTorch headers) into a shared library
that is loaded with ctypes, so a user kernel compiles in seconds; its entry
points are ``extern "C"`` functions taking plain integers and pointers.
"""
import ctypes
import hashlib
import os
import shutil
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
INCLUDE = os.path.join(ROOT, "include")
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
              "--expt-relaxed-constexpr"]


def load_inline(name, cuda_sources, functions, cpp_sources="", build_directory=None, verbose=False,
                extra_cuda_cflags=()):
    """torch.utils.cpp_extension.load_inline with the kiwi headers on the
    include path and sm_100a code generation; builds under build/jit/<name>."""
    from torch.utils.cpp_extension import load_inline as _load_inline

    if build_directory is None:
        build_directory = os.path.join(ROOT, "build", "jit", name)
    os.makedirs(build_directory, exist_ok=True)
    return _load_inline(name=name, cpp_sources=cpp_sources, cuda_sources=cuda_sources, functions=functions,
                        extra_include_paths=[INCLUDE], extra_cuda_cflags=ARCH_FLAGS + list(extra_cuda_cflags),
                        extra_cflags=["-O3", "-std=c++17"], build_directory=build_directory, verbose=verbose)


def _nvcc():
    home = os.environ.get("CUDA_HOME") or os.environ.get("CUDA_PATH") or "/usr/local/cuda"
    cand = os.path.join(home, "bin", "nvcc")
    return cand if os.path.exists(cand) else shutil.which("nvcc")


def load_cuda(name, cuda_source, extra_cuda_cflags=(), build_directory=None, verbose=False):
    """Compile `cuda_source` (which may include the kiwi headers) for sm_100a
    into ``lib<name>.so`` with nvcc and return it as a ``ctypes.CDLL``.

    Exported functions must be ``extern "C"``; set their ``argtypes`` /
    ``restype`` on the returned library before calling them.  The build is
    skipped when the library exists and was built from the same source and
    flags (a SHA-256 of both is kept beside it).  Building needs no GPU.
    """
    if not name.replace("_", "").isalnum():
        raise ValueError("name must be alphanumeric (underscores allowed)")
    nvcc = _nvcc()
    if nvcc is None:
        raise RuntimeError("load_cuda: nvcc not found (set CUDA_HOME)")
    flags = ARCH_FLAGS + ["-Xcompiler", "-fPIC", "-shared", "-I" + INCLUDE] + list(extra_cuda_cflags)
    if build_directory is None:
        build_directory = os.path.join(ROOT, "build", "jit", name)
    os.makedirs(build_directory, exist_ok=True)
    src = os.path.join(build_directory, name + ".cu")
    lib = os.path.join(build_directory, "lib" + name + ".so")
    stamp = os.path.join(build_directory, "lib" + name + ".sha256")
    key = hashlib.sha256((cuda_source + "\0" + " ".join(flags)).encode()).hexdigest()
    fresh = os.path.exists(lib) and os.path.exists(stamp) and open(stamp).read().strip() == key
    if not fresh:
        with open(src, "w") as f:
            f.write(cuda_source)
        tmp = lib + ".tmp"
        cmd = [nvcc, *flags, "-o", tmp, src, "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if verbose or r.returncode != 0:
            print(" ".join(cmd), r.stdout, r.stderr, sep="\n")
        if r.returncode != 0:
            raise RuntimeError(f"load_cuda({name!r}): nvcc failed:\n{r.stderr[-4000:]}")
        os.replace(tmp, lib)  # atomic: a concurrent loader sees the old or the new library
        with open(stamp, "w") as f:
            f.write(key + "\n")
    return ctypes.CDLL(lib)
