"""Build of the kiwi_b200 native extension (sm_100a only).

    python setup.py build_ext --inplace        # builds kiwi_b200/_C*.so in-tree

Every CUDA source is compiled with
``-gencode arch=compute_100a,code=sm_100a -lineinfo``; passing an explicit
``-gencode`` keeps torch from adding its own architecture list.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))


def _flashinfer_cutlass():
    try:
        import flashinfer  # noqa: F401  (only used to locate the vendored CUTLASS/CuTe headers)
        p = os.path.join(os.path.dirname(flashinfer.__file__), "data", "cutlass", "include")
        return [p] if os.path.isdir(p) else []
    except Exception:
        return []


ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-DNDEBUG",
    "-Xcompiler=-fPIC",
    "-Xcompiler=-fvisibility=hidden",
]
CXX_FLAGS = ["-O3", "-std=c++17", "-DNDEBUG", "-fPIC", "-fvisibility=hidden"]


def sources():
    srcs = []
    for pat in ("csrc/*.cpp", "csrc/*.cu", "src/*/*.cpp", "src/*/*.cu"):
        srcs += sorted(glob.glob(os.path.join(ROOT, pat)))
    return [os.path.relpath(s, ROOT) for s in srcs]


ext = CUDAExtension(
    name="kiwi_b200._C",
    sources=sources(),
    include_dirs=[os.path.join(ROOT, "include")] + _flashinfer_cutlass(),
    extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
)

setup(
    name="kiwi_b200",
    version="0.1.0",
    packages=["kiwi_b200", "kiwi_b200.models", "kiwi_b200.ops", "kiwi_b200.parallel", "kiwi_b200.utils"],
    ext_modules=[ext],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
