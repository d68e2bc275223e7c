// sm_100a building blocks: mbarriers, TMA (no multicast), tcgen05 / TMEM.
//
// Every wait here is bounded: a wait that exceeds its spin budget returns
// false and the caller records an error and unwinds (freeing TMEM), so a lost
// arrival can never hang the GPU.  TMA loads here are plain tiled loads of this GPU's own memory (no cluster-wide broadcast).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "kiwi/common.hpp"

namespace kiwi::sm100 {

#if defined(__CUDACC__)

KIWI_DEV uint32_t smem_addr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

KIWI_DEV bool elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "elect.sync _|p, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(pred));
    return pred != 0;
}

// ---- mbarrier ----

KIWI_DEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

KIWI_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

KIWI_DEV void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

KIWI_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

KIWI_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

/// Bounded wait for phase `parity` of `bar`; false after ~`budget` polls.
KIWI_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t budget = 1u << 26) {
    for (uint32_t i = 0; i < budget; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
    }
    return false;
}

// ---- TMA (local tensors only; never multicast) ----

KIWI_DEV void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

/// 2-D tiled TMA load into shared memory; completes tx bytes on `bar`.
/// `x` is the innermost coordinate (elements) and must keep x * elem_size a
/// multiple of 16 bytes.
KIWI_DEV void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_addr(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y)
        : "memory");
}

// ---- cp.async (LDGSTS): per-thread asynchronous global -> shared copies ----

KIWI_DEV void cp_async_16(void* smem_dst, const void* gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem_dst)), "l"(gmem_src) : "memory");
}

KIWI_DEV void cp_async_4(void* smem_dst, const void* gmem_src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(smem_dst)), "l"(gmem_src) : "memory");
}

KIWI_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

/// Waits until at most N of this thread's committed cp.async groups are pending.
template <int N>
KIWI_DEV void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

/// Makes this thread's generic-proxy shared-memory writes visible to the async
/// proxy (tcgen05.mma operand reads) before it signals an mbarrier.
KIWI_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---- tcgen05 / TMEM ----

/// Allocates `ncols` TMEM columns (power of two >= 32); the address lands in *smem_slot.
/// Whole warp.
KIWI_DEV void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(smem_slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

KIWI_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

KIWI_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
KIWI_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

/// Shared-memory matrix descriptor for a K-major, 128-byte-swizzled tile whose
/// 8-row x 128-byte swizzle atoms are stacked densely (stride 1024 bytes), as
/// a TMA load with CU_TENSOR_MAP_SWIZZLE_128B writes it.  Bits: start address
/// >> 4 [0,14), leading offset >> 4 [16,30) (unused for swizzled K-major, 1),
/// stride offset >> 4 [32,46), version 1 [46,48), layout SWIZZLE_128B = 2 [61,64).
KIWI_DEV uint64_t sw128_kmajor_desc(const void* smem_tile) {
    const uint64_t addr = smem_addr(smem_tile);
    uint64_t d = 0;
    d |= (addr >> 4) & 0x3FFFull;
    d |= static_cast<uint64_t>(1) << 16;           // LBO (16 B)
    d |= static_cast<uint64_t>(1024 >> 4) << 32;   // SBO = 1024 B between 8-row groups
    d |= static_cast<uint64_t>(1) << 46;           // descriptor version (sm100)
    d |= static_cast<uint64_t>(2) << 61;           // SWIZZLE_128B
    return d;
}

/// Same for a K-major tile of 64-byte rows (32 bf16 of K) as a TMA load with
/// CU_TENSOR_MAP_SWIZZLE_64B writes it: 8-row groups 512 B apart, layout
/// SWIZZLE_64B = 4 (the canonical K-major B64 layout
/// Swizzle<2,4,3> o ((8,m),2):((4,SBO),1) in 16-byte units).
KIWI_DEV uint64_t sw64_kmajor_desc(const void* smem_tile) {
    const uint64_t addr = smem_addr(smem_tile);
    uint64_t d = 0;
    d |= (addr >> 4) & 0x3FFFull;
    d |= static_cast<uint64_t>(1) << 16;           // LBO (16 B)
    d |= static_cast<uint64_t>(512 >> 4) << 32;    // SBO = 512 B between 8-row groups
    d |= static_cast<uint64_t>(1) << 46;           // descriptor version (sm100)
    d |= static_cast<uint64_t>(4) << 61;           // SWIZZLE_64B
    return d;
}

/// Descriptor of a K-major tile whose rows hold BK bf16 (64: 128-byte swizzle,
/// 32: 64-byte swizzle; 128: two 128-byte-swizzled 64-column sub-tiles one after
/// the other, the descriptor of the first).
template <int BK>
KIWI_DEV uint64_t kmajor_desc(const void* smem_tile) {
    static_assert(BK == 128 || BK == 64 || BK == 32, "BK must be 128, 64 or 32");
    if constexpr (BK == 32) return sw64_kmajor_desc(smem_tile);
    else return sw128_kmajor_desc(smem_tile);  // 128: the first of two 64-column sub-tiles
}

/// Instruction descriptor, kind::f16 with BF16 A/B, FP32 accumulate, both K-major.
KIWI_HD constexpr uint32_t idesc_bf16_f32(uint32_t m, uint32_t n) {
    return (1u << 4)            // D format: F32
           | (1u << 7)          // A format: BF16
           | (1u << 10)         // B format: BF16
           | ((n >> 3) << 17)   // N >> 3
           | ((m >> 4) << 24);  // M >> 4
}

/// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
KIWI_DEV void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

/// Arrives on `bar` once every tcgen05 operation this thread issued before has completed.
KIWI_DEV void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

/// Loads 32 consecutive fp32 columns of this warp's 32 TMEM lanes (one lane
/// per thread).  The wait is in the same asm statement so no use of the
/// registers can be scheduled before the load has completed.
KIWI_DEV void tmem_ld_32cols(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "{\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;\n\t}"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}


// ---- clusters of two CTAs (2-SM UMMA) ----

KIWI_DEV uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

KIWI_DEV void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

/// Cluster-window address of the same shared variable in CTA `rank` of this cluster.
KIWI_DEV uint32_t mapa(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr(p)), "r"(rank));
    return r;
}

/// Arrive (release, cluster scope) on an mbarrier given by its cluster-window address.
KIWI_DEV void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

/// 2-SM TMA load into this CTA's shared memory whose transaction bytes complete
/// on the barrier at cluster address `bar_cluster` (the pair leader's barrier).
KIWI_DEV void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster, int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_addr(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
        : "memory");
}

KIWI_DEV void tmem_alloc_pair(uint32_t* smem_slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(smem_slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

KIWI_DEV void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

/// D[tmem of both CTAs] (+)= A[smem of both] * B[smem of both]^T (M = 256 across the pair).
KIWI_DEV void mma_bf16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

/// Arrives on the barrier at cluster address `bar_cluster` (this CTA's or the
/// peer's) once every tcgen05 operation issued before by this thread completed.
KIWI_DEV void mma_commit_pair(uint32_t bar_cluster) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
                 : "memory");
}

#endif  // __CUDACC__

}  // namespace kiwi::sm100
