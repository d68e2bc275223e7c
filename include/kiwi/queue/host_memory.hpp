// Memory the queues live in.
//
// Behaviour parity: the reference allocates its rings in ROCr
// "extended-scope fine-grained" host memory so GPU accesses are uncached
// (src/queue/host_memory.cpp:94-161 of AMDResearch/kiwi).  On B200 the ring is
// mapped pinned host memory (cudaHostAlloc Mapped|Portable): GPU stores to it
// are posted PCIe writes, GPU volatile loads always go to host memory, and the
// host reads it through its own coherent caches.  Without a CUDA device (CPU
// tests, the host-only ring benchmark) the same queues use plain aligned host
// memory, which only host threads touch.
#pragma once

#include <cstddef>

namespace kiwi::queue {

enum class MemKind : int {
    kMappedPinned = 0,  // cudaHostAlloc(Mapped|Portable); the device pointer equals the host pointer (UVA)
    kHost = 1,          // aligned_alloc; host threads only
    kDevice = 2,        // cudaMalloc
};

/// True when the CUDA runtime sees at least one device.
bool cuda_device_available();

/// Mapped pinned memory when a device is present, plain host memory otherwise.
MemKind default_host_kind();

/// Zero-filled allocation of `bytes` (rounded up to 64), 4 KB aligned for host kinds.
void* alloc_zeroed(size_t bytes, MemKind kind);
void free_memory(void* p, MemKind kind);

/// Device-visible address of a host allocation (identity under UVA).
void* device_address(void* p, MemKind kind);

}  // namespace kiwi::queue
