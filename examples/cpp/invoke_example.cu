// Standalone C++ use of kiwi::invoke: a kernel calls a host callback with
// arguments; the host runs progress() until every call arrived.
//
//   make -C examples            (builds examples/build/invoke_example)
//   examples/build/invoke_example
//
// Reference counterpart: examples/invoke/invoke_example.hip.cpp of AMDResearch/kiwi.
#include <cstdio>

#include "kiwi/invoke/invoke.hpp"

using Queue = kiwi::queue::SPSCD2HQueue;

__global__ void worker(kiwi::invoke::DeviceContext<Queue>* ctx, uint8_t cb, int n) {
    auto h = ctx->get_device_handle();
    for (int i = 0; i < n; ++i) {
        const double x = 0.5 * i;
        while (!h.invoke(cb, static_cast<int32_t>(blockIdx.x), i, x)) {
        }
    }
    ctx->save_device_handle(blockIdx.x, h);
}

int main() {
    const int blocks = 4, n = 16;
    kiwi::invoke::Context<Queue> ctx(blocks, 128);
    int calls = 0;
    double sum = 0;
    const uint8_t cb = ctx.register_callback(std::function<void(int32_t, int, double)>([&](int32_t b, int i, double x) {
        ++calls;
        sum += x + 0 * b + 0 * i;
    }));
    worker<<<blocks, 32>>>(ctx.device_context(), cb, n);
    while (calls < blocks * n) ctx.progress_all();
    KIWI_CUDA_CHECK(cudaDeviceSynchronize());
    ctx.check_device_errors();
    std::printf("%d callbacks, sum %.1f (expected %.1f)\n", calls, sum, blocks * 0.5 * n * (n - 1) / 2);
    return calls == blocks * n ? 0 : 1;
}
