"""Invoke throughput through each frontend (reference: the cross-frontend
harnesses of benchmarks/invoke/frontends and benchmarks/frontends of
AMDResearch/kiwi, which run one host harness against C++, Triton and FlyDSL
kernels).

    python benchmarks/bench_frontends.py [--endpoints 8] [--msgs 20000]

* cpp:          the prebuilt kernel of the native bench module
* torch_inline: the same loop written as user CUDA and compiled at run time
                through kiwi_b200.utils.build.load_inline (the PyTorch-level
                frontend), pushing to a native counting callback
* python_cb:    the load_inline kernel with a Python callback (GIL in the loop)
Each row: messages/s over the longer of the device push time (first push to
last, %globaltimer) and the host time until the callback has seen every
message, 8-byte payloads, one warp per endpoint, native progress threads.
"""
import argparse
import json
import os
import sys
import time

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import torch  # noqa: E402

import kiwi_b200  # noqa: E402
from kiwi_b200 import invoke  # noqa: E402
from kiwi_b200.utils.build import load_inline  # noqa: E402

# The CUDA source takes raw device addresses, so nvcc never parses the torch
# headers (the generated C++ wrapper is the only torch-dependent part).
CUDA = r"""
#include <cstdint>
#include <kiwi/invoke/device_context.cuh>
#include <kiwi/queue/queue.hpp>
#include <kiwi/ptx.cuh>

using Ctx = kiwi::invoke::DeviceContext<kiwi::queue::SPSCD2HQueue>;

__global__ void push_kernel(Ctx* ctx, uint8_t cb, uint32_t msgs, unsigned long long* t, uint32_t* status) {
    auto h = ctx->get_device_handle();
    if (blockIdx.x == 0 && threadIdx.x == 0) t[0] = kiwi::ptx::globaltimer();
    for (uint32_t i = 0; i < msgs; ++i) {
        const uint64_t w = (static_cast<uint64_t>(blockIdx.x) << 32) | i;
        kiwi::ptx::Deadline dl(2000000000ull);
        while (!h.invoke(cb, w)) {
            if (dl.expired()) {
                if (threadIdx.x == 0) status[0] = 1;
                ctx->save_device_handle(blockIdx.x, h);
                return;
            }
        }
    }
    ctx->save_device_handle(blockIdx.x, h);
    __syncwarp();
    if (threadIdx.x == 0) atomicMax(&t[1], static_cast<unsigned long long>(kiwi::ptx::globaltimer()));
}

void push(int64_t ctx_ptr, int64_t cb, int64_t endpoints, int64_t msgs, int64_t t_ptr, int64_t status_ptr) {
    push_kernel<<<endpoints, 32>>>(reinterpret_cast<Ctx*>(ctx_ptr), static_cast<uint8_t>(cb),
                                   static_cast<uint32_t>(msgs), reinterpret_cast<unsigned long long*>(t_ptr),
                                   reinterpret_cast<uint32_t*>(status_ptr));
}
"""
CPP = "void push(int64_t ctx_ptr, int64_t cb, int64_t endpoints, int64_t msgs, int64_t t_ptr, int64_t status_ptr);"


def frontend_run(mod, endpoints, msgs, threads, python_cb=False, timeout_s=30.0):
    ctx = invoke.Context(num_endpoints=endpoints, capacity=1024)
    if python_cb:
        box = [0]

        def on_msg(word):
            box[0] += 1

        cb = ctx.register_callback(on_msg, "<Q")
        count = lambda: box[0]  # noqa: E731
    else:
        cb = ctx._ctx.register_native_counter()
        count = lambda: ctx._ctx.native_count  # noqa: E731
    ctx.start(num_threads=threads)
    t = torch.zeros(2, dtype=torch.int64, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    h0 = time.perf_counter()
    mod.push(ctx.device_context_ptr, cb, endpoints, msgs, t.data_ptr(), status.data_ptr())
    want = endpoints * msgs
    end = time.time() + timeout_s
    while count() < want and time.time() < end:
        time.sleep(1e-4)
    host_s = time.perf_counter() - h0
    torch.cuda.synchronize()
    got = count()
    ctx.stop()
    ctx.check_device_errors()
    dev_s = int(t[1].item() - t[0].item()) / 1e9
    span = max(dev_s, host_s)
    return {"messages": got, "ok": got == want and int(status.item()) == 0,
            "msgs_per_s": got / span if span > 0 else 0.0, "device_s": dev_s, "host_s": host_s}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--endpoints", type=int, default=8)
    ap.add_argument("--msgs", type=int, default=20000)
    ap.add_argument("--threads", type=int, default=2)
    args = ap.parse_args()
    C = kiwi_b200.native()
    rows = []
    r = C.bench.invoke_throughput(endpoints=args.endpoints, threads=args.threads, msgs_per_endpoint=args.msgs,
                                  payload_bytes=8)
    rows.append({"frontend": "cpp", "messages": r["messages"], "ok": bool(r["ok"]),
                 "msgs_per_s": r["messages"] / (r["device_ns"] / 1e9) if r["device_ns"] else 0.0})
    mod = load_inline("kiwi_bench_frontends", [CUDA], ["push"], cpp_sources=[CPP])
    rows.append({"frontend": "torch_inline", **frontend_run(mod, args.endpoints, args.msgs, args.threads)})
    rows.append({"frontend": "python_cb", **frontend_run(mod, args.endpoints, max(1, args.msgs // 4), args.threads,
                                                         python_cb=True)})
    for row in rows:
        print("RESULT " + json.dumps({"bench": "invoke_frontends", "endpoints": args.endpoints, **row}), flush=True)


if __name__ == "__main__":
    main()
