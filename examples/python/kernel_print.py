"""A CUDA kernel prints through a native C++ callback (no Python in the loop).

    python examples/python/kernel_print.py [-n 8]

The kernel invokes a callback with (int32 step, float value, uint64 tag); the
callback is registered with ``Context.register_native_print``, so the progress
loop formats and prints each line in C++.  (Reference counterpart: the
Triton/FlyDSL print examples with their shared C++ extension,
examples/triton/triton_print_example.py and examples/common/kiwi_print_ext.hip.cpp
of AMDResearch/kiwi.)
"""
import argparse
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
import torch  # noqa: E402

from kiwi_b200 import invoke  # noqa: E402
from kiwi_b200.utils.build import load_inline  # noqa: E402

CUDA = r"""
#include <cstdint>
#include <kiwi/invoke/device_context.cuh>
#include <kiwi/queue/queue.hpp>

using Ctx = kiwi::invoke::DeviceContext<kiwi::queue::SPSCD2HQueue>;

__global__ void print_kernel(Ctx* ctx, uint8_t cb, int n) {
    auto h = ctx->get_device_handle();            // one warp owns endpoint 0
    for (int i = 0; i < n; ++i) {
        const int32_t step = i;
        const float value = 0.5f * i;
        const uint64_t tag = 0xC0FFEE00ull + i;
        while (!h.invoke(cb, step, value, tag)) {}
    }
    ctx->save_device_handle(blockIdx.x, h);       // a later launch continues from here
}

void run_print(int64_t ctx_ptr, int64_t cb, int64_t n) {
    print_kernel<<<1, 32>>>(reinterpret_cast<Ctx*>(ctx_ptr), static_cast<uint8_t>(cb), static_cast<int>(n));
}
"""
CPP = "void run_print(int64_t ctx_ptr, int64_t cb, int64_t n);"


def main(n=8):
    mod = load_inline("kiwi_example_print", [CUDA], ["run_print"], cpp_sources=[CPP])
    ctx = invoke.Context(num_endpoints=1, capacity=1024)
    cb = ctx.register_native_print("[C++ callback] step=%d value=%.2f tag=0x%llx", "<ifQ")
    mod.run_print(ctx.device_context_ptr, cb, n)
    executed = 0
    while executed < n:
        executed += ctx.progress(0)
    torch.cuda.synchronize()
    ctx.check_device_errors()
    return executed


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("-n", type=int, default=8, help="number of invokes")
    args = ap.parse_args()
    print(f"the kernel invoked the C++ print callback {main(args.n)} times")
