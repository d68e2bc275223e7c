// kiwi::p2p device API: put / get / signal / wait straight into peer GPUs'
// memory over NVLink 5, plus NVLS multimem broadcast and reduction.
//
// Parity with the reference's GPU-side P2P (AMDResearch/kiwi): post_p,
// post_put + readiness byte, poll_counter (apps/p2p/context.hip.hpp:54-251,
// readiness.hip.hpp:10-31, comp_counter.hip.hpp:47-86).  The reference posts
// descriptors to a CPU proxy that issues RDMA; here the kernel stores into the
// peer's heap itself (the host/queue path carries control only), so:
//   put      = warp- or block-cooperative 16-byte stores to the peer mapping
//   signal   = st.release.sys / red.release.sys.add on the peer's flag word
//   wait     = ld.acquire.sys polling with a deadline (never unbounded)
//   put_ll8  = small messages whose 8-byte words carry data + sequence (no fence)
//   get      = 16-byte loads from the peer mapping
// Checked mode (HeapView::check set by SymmetricHeap::set_checks): each call
// validates its range first and records and skips a bad one, never traps.
// Ordering: a signal issued after __syncwarp()/__syncthreads() releases every
// store the warp/block made before it (PTX release is cumulative over writes
// the releasing thread has observed through the barrier).
#pragma once

#include "kiwi/p2p/heap.hpp"
#include "kiwi/ptx.cuh"

namespace kiwi::p2p {

enum class SignalOp : int { kSet = 0, kAdd = 1 };
enum class Cmp : int { kEq = 0, kGe = 1, kNe = 2 };

#if defined(__CUDACC__)

KIWI_DEV uint8_t* remote(const HeapView& h, int rank, uint64_t off) { return h.base[rank] + off; }

/// Checked mode (HeapView::check non-null): false, with the first violation
/// recorded, when the access leaves [0, check_limit) of a valid rank's heap.
/// Every lane of a cooperative call computes the same answer, so a rejected
/// put or get is skipped by the whole warp or block.
KIWI_DEV bool access_ok(const HeapView& h, int rank, uint64_t off, uint64_t bytes, CheckSite site) {
    if (h.check == nullptr) return true;
    if (heap_range_ok(h.world, h.check_limit, rank, off, bytes)) return true;
    if (atomicCAS(h.check, 0u, 1u) == 0u) {
        h.check[1] = static_cast<uint32_t>(site);
        h.check[2] = static_cast<uint32_t>(rank);
        h.check[3] = static_cast<uint32_t>(off);
        __threadfence_system();
    }
    return false;
}

/// Copies `bytes` from src to dst with `nthreads` cooperating threads
/// (thread index `tid`).  Both addresses 16-byte aligned for the vector part;
/// a tail of < 16 bytes goes byte by byte.  4 independent 16-byte loads are in
/// flight per thread to cover NVLink latency.
KIWI_DEV void coop_copy(void* dst, const void* src, uint64_t bytes, uint32_t tid, uint32_t nthreads) {
    const uint64_t nvec = bytes / 16;
    uint4* d = static_cast<uint4*>(dst);
    const uint4* s = static_cast<const uint4*>(src);
    uint64_t i = tid;
    for (; i + 3 * static_cast<uint64_t>(nthreads) < nvec; i += 4 * static_cast<uint64_t>(nthreads)) {
        const uint4 a = ptx::ld_v4(s + i);
        const uint4 b = ptx::ld_v4(s + i + nthreads);
        const uint4 c = ptx::ld_v4(s + i + 2 * static_cast<uint64_t>(nthreads));
        const uint4 e = ptx::ld_v4(s + i + 3 * static_cast<uint64_t>(nthreads));
        ptx::st_v4(d + i, a);
        ptx::st_v4(d + i + nthreads, b);
        ptx::st_v4(d + i + 2 * static_cast<uint64_t>(nthreads), c);
        ptx::st_v4(d + i + 3 * static_cast<uint64_t>(nthreads), e);
    }
    for (; i < nvec; i += nthreads) ptx::st_v4(d + i, ptx::ld_v4(s + i));
    const uint64_t tail = bytes - nvec * 16;
    if (tail && tid < tail) {
        static_cast<uint8_t*>(dst)[nvec * 16 + tid] = static_cast<const uint8_t*>(src)[nvec * 16 + tid];
    }
}

/// Warp-cooperative put of `bytes` from local `src` into rank's heap at `dst_off`.
KIWI_DEV void put_warp(const HeapView& h, int rank, uint64_t dst_off, const void* src, uint64_t bytes) {
    if (!access_ok(h, rank, dst_off, bytes, kCheckPut)) return;
    coop_copy(remote(h, rank, dst_off), src, bytes, ptx::lane_id(), 32);
}

/// Block-cooperative put.
KIWI_DEV void put_block(const HeapView& h, int rank, uint64_t dst_off, const void* src, uint64_t bytes) {
    if (!access_ok(h, rank, dst_off, bytes, kCheckPut)) return;
    coop_copy(remote(h, rank, dst_off), src, bytes, threadIdx.x, blockDim.x);
}

/// Warp-cooperative get of `bytes` from rank's heap at `src_off` into local `dst`.
KIWI_DEV void get_warp(const HeapView& h, int rank, uint64_t src_off, void* dst, uint64_t bytes) {
    if (!access_ok(h, rank, src_off, bytes, kCheckGet)) return;
    coop_copy(dst, remote(h, rank, src_off), bytes, ptx::lane_id(), 32);
}

KIWI_DEV void get_block(const HeapView& h, int rank, uint64_t src_off, void* dst, uint64_t bytes) {
    if (!access_ok(h, rank, src_off, bytes, kCheckGet)) return;
    coop_copy(dst, remote(h, rank, src_off), bytes, threadIdx.x, blockDim.x);
}

/// Signals a 64-bit flag in rank's heap with release semantics (system scope).
/// Call from one thread after a warp/block barrier that follows the puts.
KIWI_DEV void signal(const HeapView& h, int rank, uint64_t flag_off, uint64_t value, SignalOp op) {
    if (!access_ok(h, rank, flag_off, sizeof(uint64_t), kCheckSignal)) return;
    void* f = remote(h, rank, flag_off);
    if (op == SignalOp::kSet) {
        ptx::st_release_sys_u64(f, value);
    } else {
        ptx::red_release_sys_add_u64(f, value);
    }
}

KIWI_DEV bool cmp_ok(uint64_t v, Cmp c, uint64_t want) {
    switch (c) {
        case Cmp::kEq: return v == want;
        case Cmp::kGe: return v >= want;
        case Cmp::kNe: return v != want;
    }
    return false;
}

/// Waits (one thread) until *flag satisfies `c` against `want`, or the
/// deadline passes (returns kTimeout; the caller decides what to record).
/// Polls with ld.acquire.sys.  Measured on B200 over NVLink: a system-scope
/// fence costs ~1.5 us, so relaxed polls followed by one fence.acq_rel.sys were
/// slower (4.7 us one-way put) than acquire polls (3.2 us).
KIWI_DEV Status wait(const uint64_t* flag, Cmp c, uint64_t want, uint64_t timeout_ns) {
    if (cmp_ok(ptx::ld_acquire_sys_u64(flag), c, want)) return Status::kOk;
    ptx::Deadline dl(timeout_ns);
    while (!cmp_ok(ptx::ld_acquire_sys_u64(flag), c, want)) {
        if (dl.expired()) return Status::kTimeout;
    }
    return Status::kOk;
}

// ---- LL8 small-message path: every 8-byte word carries 4 data bytes and a
// 32-bit sequence number, so a receiver that sees the sequence in a word sees
// its data; no fence or flag is needed (8-byte single-copy atomicity only).

/// Warp-cooperative LL8 put of `nwords` 32-bit words into rank's heap at dst_off
/// (8 bytes per word on the wire).
KIWI_DEV void put_ll8_warp(const HeapView& h, int rank, uint64_t dst_off, const uint32_t* src, uint32_t nwords,
                           uint32_t seq) {
    if (!access_ok(h, rank, dst_off, 8ull * nwords, kCheckLl8)) return;
    uint64_t* dst = reinterpret_cast<uint64_t*>(h.base[rank] + dst_off);
    for (uint32_t i = ptx::lane_id(); i < nwords; i += 32) {
        ptx::st_volatile_u64(dst + i, static_cast<uint64_t>(src[i]) | (static_cast<uint64_t>(seq) << 32));
    }
}

/// Warp-cooperative LL8 receive: waits until every word of the local buffer
/// carries `seq`, copying the data words to `out`.  Returns kTimeout on expiry.
KIWI_DEV Status recv_ll8_warp(const uint64_t* local, uint32_t* out, uint32_t nwords, uint32_t seq,
                              uint64_t timeout_ns) {
    bool ok = true;
    for (uint32_t i = ptx::lane_id(); i < nwords; i += 32) {
        ptx::Deadline dl(timeout_ns);
        uint64_t v = ptx::ld_volatile_u64(local + i);
        while (static_cast<uint32_t>(v >> 32) != seq) {
            if (dl.expired()) {
                ok = false;
                break;
            }
            v = ptx::ld_volatile_u64(local + i);
        }
        if (!ok) break;
        out[i] = static_cast<uint32_t>(v);
    }
    return __all_sync(ptx::kFullMask, ok) ? Status::kOk : Status::kTimeout;
}

// ---- NVLS multimem (one instruction reaches every rank bound to the object) ----

/// Stores 16 bytes to the same offset of every rank's heap.
KIWI_DEV void mc_store_v4(void* mc_addr, uint4 v) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc_addr), "r"(v.x),
                 "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

/// Loads 4 fp32 from every rank's heap at this offset and returns their sum.
KIWI_DEV float4 mc_reduce_add_f32_v4(const void* mc_addr) {
    float4 r;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
                 : "l"(mc_addr)
                 : "memory");
    return r;
}

/// Loads 8 bf16 (as 4 bf16x2) from every rank and returns their sum (fp32 accumulate in the switch).
KIWI_DEV uint4 mc_reduce_add_bf16x8(const void* mc_addr) {
    uint4 r;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(mc_addr)
                 : "memory");
    return r;
}

/// Adds to a 64-bit counter on every rank (multicast release reduction).
KIWI_DEV void mc_red_add_u64(void* mc_addr, uint64_t v) {
    asm volatile("multimem.red.release.sys.global.add.u64 [%0], %1;" ::"l"(mc_addr), "l"(v) : "memory");
}

/// Block-cooperative broadcast of `bytes` (16-byte multiple) from local src to
/// every rank's heap at mc_off.
KIWI_DEV void mc_broadcast_block(const HeapView& h, uint64_t mc_off, const void* src, uint64_t bytes) {
    if (!access_ok(h, h.rank, mc_off, bytes, kCheckMulticast)) return;
    const uint4* s = static_cast<const uint4*>(src);
    uint4* d = reinterpret_cast<uint4*>(h.mc + mc_off);
    for (uint64_t i = threadIdx.x; i < bytes / 16; i += blockDim.x) mc_store_v4(d + i, ptx::ld_v4(s + i));
}

#endif  // __CUDACC__

}  // namespace kiwi::p2p
