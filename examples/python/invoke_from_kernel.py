"""A user CUDA kernel calls Python from the GPU through kiwi_b200.invoke.

    python examples/python/invoke_from_kernel.py [--fast-build]

Each block of the kernel reports (block id, reading) to a Python callback
through its own invoke endpoint while it runs; a native progress thread pinned
near the GPU dispatches the messages.  (Reference counterpart:
examples/invoke/invoke_example.hip.cpp and the Triton/FlyDSL print examples of
AMDResearch/kiwi.)  ``--fast-build`` compiles the kernel with nvcc alone and
loads it with ctypes (``kiwi_b200.utils.build.load_cuda``) instead of building a
PyTorch extension, which takes seconds instead of about a minute.
"""
import argparse
import ctypes
import os
import sys
import threading

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
import torch  # noqa: E402

from kiwi_b200 import invoke  # noqa: E402
from kiwi_b200.utils.build import load_cuda, load_inline  # noqa: E402

CUDA = r"""
#include <cstdint>
#include <kiwi/invoke/device_context.cuh>
#include <kiwi/queue/queue.hpp>

using Ctx = kiwi::invoke::DeviceContext<kiwi::queue::SPSCD2HQueue>;

__global__ void sensor_kernel(Ctx* ctx, uint8_t cb, int readings) {
    auto h = ctx->get_device_handle();            // endpoint = blockIdx.x
    for (int i = 0; i < readings; ++i) {
        const float value = blockIdx.x * 100.0f + i;
        while (!h.invoke(cb, static_cast<uint32_t>(blockIdx.x), value)) {}
    }
    ctx->save_device_handle(blockIdx.x, h);
}

void run_sensors(int64_t ctx_ptr, int64_t cb, int64_t blocks, int64_t readings) {
    sensor_kernel<<<blocks, 32>>>(reinterpret_cast<Ctx*>(ctx_ptr), static_cast<uint8_t>(cb),
                                  static_cast<int>(readings));
}

// The same entry point with C linkage, for the ctypes build.
extern "C" void kiwi_run_sensors(int64_t ctx_ptr, int64_t cb, int64_t blocks, int64_t readings) {
    run_sensors(ctx_ptr, cb, blocks, readings);
}
"""
CPP = "void run_sensors(int64_t ctx_ptr, int64_t cb, int64_t blocks, int64_t readings);"


def build(fast=False):
    """A callable run_sensors(ctx_ptr, cb, blocks, readings)."""
    if fast:
        lib = load_cuda("kiwi_example_sensors_c", CUDA)
        lib.kiwi_run_sensors.argtypes = [ctypes.c_int64] * 4
        lib.kiwi_run_sensors.restype = None
        return lib.kiwi_run_sensors
    return load_inline("kiwi_example_sensors", [CUDA], ["run_sensors"], cpp_sources=[CPP]).run_sensors


def main(blocks=4, readings=8, fast=False):
    run_sensors = build(fast)
    ctx = invoke.Context(num_endpoints=blocks, capacity=256)
    got = []
    lock = threading.Lock()

    def on_reading(block, value):
        with lock:
            got.append((block, value))

    cb = ctx.register_callback(on_reading, "<If")
    ctx.start(num_threads=1)
    run_sensors(ctx.device_context_ptr, cb, blocks, readings)
    torch.cuda.synchronize()
    ctx.stop()
    ctx.check_device_errors()
    return got


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--fast-build", action="store_true", help="nvcc + ctypes instead of a PyTorch extension")
    readings = main(fast=ap.parse_args().fast_build)
    print(f"{len(readings)} readings from the GPU, e.g. {sorted(readings)[:3]}")
