#include "kiwi/queue/host_memory.hpp"

#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>

#include "kiwi/common.hpp"

namespace kiwi::queue {

bool cuda_device_available() {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return n > 0;
}

MemKind default_host_kind() {
    static const MemKind kind = cuda_device_available() ? MemKind::kMappedPinned : MemKind::kHost;
    return kind;
}

void* alloc_zeroed(size_t bytes, MemKind kind) {
    bytes = round_up(bytes == 0 ? 64 : bytes, 64);
    void* p = nullptr;
    switch (kind) {
        case MemKind::kMappedPinned:
            KIWI_CUDA_CHECK(cudaHostAlloc(&p, bytes, cudaHostAllocMapped | cudaHostAllocPortable));
            std::memset(p, 0, bytes);
            return p;
        case MemKind::kHost:
            p = std::aligned_alloc(4096, round_up(bytes, 4096));
            if (!p) throw kiwi::error("kiwi::queue: host allocation failed");
            std::memset(p, 0, bytes);
            return p;
        case MemKind::kDevice:
            KIWI_CUDA_CHECK(cudaMalloc(&p, bytes));
            KIWI_CUDA_CHECK(cudaMemset(p, 0, bytes));
            return p;
    }
    return nullptr;
}

void free_memory(void* p, MemKind kind) {
    if (!p) return;
    switch (kind) {
        case MemKind::kMappedPinned: cudaFreeHost(p); break;
        case MemKind::kHost: std::free(p); break;
        case MemKind::kDevice: cudaFree(p); break;
    }
}

void* device_address(void* p, MemKind kind) {
    if (kind != MemKind::kMappedPinned || p == nullptr) return p;
    void* d = nullptr;
    KIWI_CUDA_CHECK(cudaHostGetDevicePointer(&d, p, 0));
    return d;
}

}  // namespace kiwi::queue
