// Device memory-model and warp primitives for sm_100a, written as inline PTX.
//
// Counterparts of the reference's GCN helpers (apps/ep/memory_scope.hip.hpp:23-134,
// include/kiwi/queue/detail/chunk.hip.hpp:149-198 of AMDResearch/kiwi):
//   readfirstlane / wave_uniform  -> __shfl_sync(full, v, 0)
//   s_sleep                       -> __nanosleep
//   sc0 sc1 system-scope ld/st    -> ld.acquire.sys / st.release.sys / ld.volatile / st.volatile
//   wall_clock64                  -> %globaltimer (ns)
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "kiwi/common.hpp"

namespace kiwi::ptx {

inline constexpr unsigned kFullMask = 0xffffffffu;

KIWI_DEV uint32_t lane_id() {
    uint32_t l;
    asm volatile("mov.u32 %0, %%laneid;" : "=r"(l));
    return l;
}

KIWI_DEV uint32_t warp_id_in_block() { return threadIdx.x / 32; }

KIWI_DEV uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

KIWI_DEV uint64_t clock64() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%clock64;" : "=l"(t));
    return t;
}

template <typename T>
KIWI_DEV T bcast(T v, int src = 0) {
    return __shfl_sync(kFullMask, v, src);
}

KIWI_DEV uint64_t bcast64(uint64_t v, int src = 0) {
    const uint32_t lo = __shfl_sync(kFullMask, static_cast<uint32_t>(v), src);
    const uint32_t hi = __shfl_sync(kFullMask, static_cast<uint32_t>(v >> 32), src);
    return (static_cast<uint64_t>(hi) << 32) | lo;
}

/// Exclusive prefix sum over the warp; `total` receives the warp-wide sum.
KIWI_DEV uint32_t warp_exclusive_scan(uint32_t v, uint32_t& total) {
    const uint32_t lane = lane_id();
    uint32_t x = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const uint32_t y = __shfl_up_sync(kFullMask, x, d);
        if (lane >= static_cast<uint32_t>(d)) x += y;
    }
    total = __shfl_sync(kFullMask, x, 31);
    return x - v;
}

// ---- volatile (relaxed, system-visible) accesses, used on mapped host memory ----

KIWI_DEV void st_volatile_v4(void* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b),
                 "r"(c), "r"(d)
                 : "memory");
}

KIWI_DEV uint4 ld_volatile_v4(const void* p) {
    uint4 v;
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}

KIWI_DEV uint64_t ld_volatile_u64(const void* p) {
    uint64_t v;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

KIWI_DEV uint32_t ld_volatile_u32(const void* p) {
    uint32_t v;
    asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

KIWI_DEV void st_volatile_u64(void* p, uint64_t v) {
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

KIWI_DEV void st_volatile_u32(void* p, uint32_t v) {
    asm volatile("st.volatile.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// ---- acquire / release at system scope (peer GPUs over NVLink, host) ----

KIWI_DEV uint64_t ld_acquire_sys_u64(const void* p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

KIWI_DEV uint32_t ld_acquire_sys_u32(const void* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

KIWI_DEV uint32_t ld_acquire_gpu_u32(const void* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

KIWI_DEV uint64_t ld_acquire_gpu_u64(const void* p) {
    uint64_t v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

KIWI_DEV uint64_t ld_relaxed_sys_u64(const void* p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

KIWI_DEV uint32_t ld_relaxed_sys_u32(const void* p) {
    uint32_t v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

KIWI_DEV void st_release_sys_u64(void* p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

KIWI_DEV void st_release_sys_u32(void* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

KIWI_DEV void st_release_gpu_u32(void* p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

KIWI_DEV void st_relaxed_sys_u64(void* p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

KIWI_DEV void red_release_sys_add_u64(void* p, uint64_t v) {
    asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

KIWI_DEV void red_release_sys_add_u32(void* p, uint32_t v) {
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

KIWI_DEV void red_release_gpu_add_u32(void* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

KIWI_DEV uint32_t atom_add_acq_rel_gpu_u32(void* p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

KIWI_DEV void fence_sys() { asm volatile("fence.sc.sys;" ::: "memory"); }
KIWI_DEV void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
KIWI_DEV void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
/// Orders generic-proxy writes (st, P2P stores that landed) before later
/// async-proxy reads (TMA) of the same memory.
KIWI_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// ---- 16-byte vector copies (P2P data plane) ----

KIWI_DEV uint4 ld_v4(const void* p) {
    uint4 v;
    asm volatile("ld.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

KIWI_DEV uint4 ld_nc_v4(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

KIWI_DEV void st_v4(void* p, uint4 v) {
    asm volatile("st.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}

/// Store that bypasses L1 allocation and is marked streaming (evict-first).
KIWI_DEV void st_cs_v4(void* p, uint4 v) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}

/// Bounded wait helper: `expired()` is checked every `check_every` spins so the
/// timer read stays off the hot path.
struct Deadline {
    uint64_t end_ns;
    uint32_t spins;
    KIWI_DEV explicit Deadline(uint64_t timeout_ns) : end_ns(globaltimer() + timeout_ns), spins(0) {}
    KIWI_DEV bool expired() {
        if ((++spins & 63u) != 0) return false;
        return globaltimer() > end_ns;
    }
};

}  // namespace kiwi::ptx
