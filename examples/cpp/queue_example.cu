// Standalone C++ use of kiwi::queue: each warp of a kernel pushes messages
// into its own GPU->host ring (SPSC, one warp per ring); the host pops them.
//
//   make -C examples            (builds examples/build/queue_example)
//   examples/build/queue_example
//
// Reference counterpart: examples/simple_example of AMDResearch/kiwi.
#include <cstdio>
#include <cstring>
#include <vector>

#include "kiwi/queue/queue.hpp"

using kiwi::queue::SPSCD2HQueue;
using kiwi::queue::SpscD2HHandle;

struct Reading {
    uint32_t block;
    uint32_t step;
    float value;
    uint32_t pad;
};

__global__ void producer(SpscD2HHandle* handles, int steps) {
    SpscD2HHandle h = handles[blockIdx.x];          // by value: the producer position lives in registers
    for (int i = 0; i < steps; ++i) {
        const Reading r{blockIdx.x, static_cast<uint32_t>(i), 0.25f * i, 0};
        while (!h.push_reg(r, /*metadata=*/blockIdx.x)) {   // warp-collective; false while the ring is full
        }
    }
}

int main() {
    const int blocks = 4, steps = 1000;
    std::vector<SPSCD2HQueue*> queues;
    std::vector<SpscD2HHandle> host_handles;
    for (int b = 0; b < blocks; ++b) {
        queues.push_back(new SPSCD2HQueue(64));     // 64 lines: the producers wait for the host often
        host_handles.push_back(queues.back()->device_handle());
    }
    SpscD2HHandle* handles = nullptr;
    KIWI_CUDA_CHECK(cudaMalloc(&handles, blocks * sizeof(SpscD2HHandle)));
    KIWI_CUDA_CHECK(cudaMemcpy(handles, host_handles.data(), blocks * sizeof(SpscD2HHandle), cudaMemcpyHostToDevice));
    producer<<<blocks, 32>>>(handles, steps);
    KIWI_CUDA_CHECK(cudaGetLastError());
    std::vector<int> next(blocks, 0);
    int got = 0, bad = 0;
    alignas(16) uint8_t buf[kiwi::queue::kMaxMessageBytes];
    while (got < blocks * steps) {
        for (int b = 0; b < blocks; ++b) {
            uint32_t meta = 0, bytes = 0;
            while (queues[b]->try_pop(buf, &meta, &bytes)) {
                Reading r;
                std::memcpy(&r, buf, sizeof(r));
                if (bytes != sizeof(Reading) || meta != static_cast<uint32_t>(b) || r.block != static_cast<uint32_t>(b) ||
                    r.step != static_cast<uint32_t>(next[b])) {
                    ++bad;
                }
                ++next[b];
                ++got;
            }
        }
    }
    KIWI_CUDA_CHECK(cudaDeviceSynchronize());
    for (auto* q : queues) {
        const auto e = q->error();
        if (e.code) ++bad;
        delete q;
    }
    cudaFree(handles);
    std::printf("%d messages from %d warps, %d out of order or damaged\n", got, blocks, bad);
    return bad == 0 ? 0 : 1;
}
