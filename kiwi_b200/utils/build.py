"""Build helpers for user CUDA code that uses the kiwi headers.

``load_inline(name, cuda_sources, functions)`` wraps
``torch.utils.cpp_extension.load_inline`` with the repository's ``include/``
directory and sm_100a code generation, so a user kernel can
``#include <kiwi/invoke/device_context.cuh>`` and call host callbacks that a
:class:`kiwi_b200.invoke.Context` registered (pass ``ctx.device_context_ptr``
to the kernel as a ``kiwi::invoke::DeviceContext<kiwi::queue::SPSCD2HQueue>*``).
This is the PyTorch-level replacement of the reference's Triton / FlyDSL
frontends (python/kiwi_triton.py, python/kiwi_flydsl of AMDResearch/kiwi).
"""
import os

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
INCLUDE = os.path.join(ROOT, "include")
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
              "--expt-relaxed-constexpr"]


def load_inline(name, cuda_sources, functions, cpp_sources="", build_directory=None, verbose=False,
                extra_cuda_cflags=()):
    from torch.utils.cpp_extension import load_inline as _load_inline

    if build_directory is None:
        build_directory = os.path.join(ROOT, "build", "jit", name)
    os.makedirs(build_directory, exist_ok=True)
    return _load_inline(name=name, cpp_sources=cpp_sources, cuda_sources=cuda_sources, functions=functions,
                        extra_include_paths=[INCLUDE], extra_cuda_cflags=ARCH_FLAGS + list(extra_cuda_cflags),
                        extra_cflags=["-O3", "-std=c++17"], build_directory=build_directory, verbose=verbose)
