// kiwi::ep kernels: routing, fused quantise + NVLink dispatch, receive-side
// count / scatter + dequantise, combine send and combine reduce.
//
// Parity with the reference's EP kernels (AMDResearch/kiwi):
//   dispatch  apps/ep/dispatch.hip.cpp:334-993  (dedup by destination rank,
//             slot per (source rank, token), readiness per source, unpack)
//   combine   apps/ep/combine.hip.cpp:558-1033  (return rows to the source,
//             reduce over ranks)
// The reference moves rows through CPU proxies (RDMA) or HIP-IPC stores and
// leaves routing, quantisation and the expert FFN to the caller.  Here the
// dispatch kernel also routes and quantises (1x128 FP8 with fp32 scales, or
// NVFP4 16-element blocks with e4m3 scales), stores with 16-byte st.global
// straight into every destination GPU's heap over NVLink, and the receive
// side lays rows out expert-major for the tcgen05 grouped GEMM.
// Completion per round: the last CTA of a grid (atomic counter) issues a
// system-scope release store of (epoch << 32 | tokens) to every rank's flag;
// receivers wait with ld.acquire.sys under a deadline.
#include <cuda_bf16.h>
#include <cuda_fp4.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>

#include "kiwi/ep/debug_timing.hpp"
#include "kiwi/ep/kernels.hpp"
#include "kiwi/ep/quant.cuh"
#include "kiwi/ptx.cuh"

namespace kiwi::ep {

namespace {

constexpr int kThreads = 256;
constexpr int kDispatchRaw = 3;  // dispatch_kernel mode: caller-quantised rows travel as bytes

KIWI_DEV void set_error(const EpWorkspace& ws, uint32_t code, uint32_t site, uint32_t info, int rank) {
    if (atomicCAS(&ws.error[0], 0u, code) == 0u) {
        ws.error[1] = site;
        ws.error[2] = info;
        ws.error[3] = static_cast<uint32_t>(rank);
    }
}

KIWI_DEV const uint8_t* meta_ptr(const EpConfig& c, const uint8_t* base, uint64_t slot) {
    return base + c.meta_off(slot);
}

/// Loads 16 bytes that a peer GPU stored into this GPU's memory: L2 only
/// (.cg), never a possibly stale L1 line.
KIWI_DEV uint4 ld_cg_v4(const void* p) {
    uint4 v;
    asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
KIWI_DEV uint2 ld_cg_v2(const void* p) {
    uint2 v;
    asm volatile("ld.global.cg.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}
KIWI_DEV uint32_t ld_cg_u32(const void* p) {
    uint32_t v;
    asm volatile("ld.global.cg.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
KIWI_DEV float ld_cg_f32(const void* p) { return __uint_as_float(ld_cg_u32(p)); }

/// Last-CTA completion: after every CTA has issued its stores, the last one
/// to arrive publishes `value` to flag offset `flag_off` on every rank.
KIWI_DEV void grid_done_signal(const EpConfig& c, const p2p::HeapView& h, uint32_t* counter, uint64_t flag_off,
                               uint64_t value) {
    __syncthreads();
    if (threadIdx.x == 0) {
        ptx::fence_sys();
        const uint32_t prev = atomicAdd(counter, 1u);
        if (prev == gridDim.x - 1) {
            ptx::fence_sys();
            for (int r = 0; r < c.world; ++r) ptx::st_release_sys_u64(h.base[r] + flag_off, value);
            *reinterpret_cast<volatile uint32_t*>(counter) = 0;
        }
    }
}

/// Threads [0, world) wait until every rank's flag at `flag_of(src)` carries
/// `epoch`; returns false (error recorded) on timeout.  Block-collective.
template <typename FlagOf>
KIWI_DEV bool wait_all_flags(const EpConfig& c, const p2p::HeapView& h, const EpWorkspace& ws, uint32_t epoch,
                             FlagOf flag_of, uint32_t site, uint64_t timeout_ns, uint32_t* tokens_out,
                             const PhaseScope& ps) {
    __shared__ int s_fail;
    if (threadIdx.x == 0) s_fail = 0;
    __syncthreads();
    if (threadIdx.x < static_cast<unsigned>(c.world)) {
        const uint64_t* f = reinterpret_cast<const uint64_t*>(h.base[h.rank] + flag_of(threadIdx.x));
        ps.wait_begin();
        ptx::Deadline dl(timeout_ns);
        uint64_t v = ptx::ld_acquire_sys_u64(f);
        while (static_cast<uint32_t>(v >> 32) != epoch) {
            if (dl.expired()) {
                set_error(ws, static_cast<uint32_t>(Status::kTimeout), site, threadIdx.x, c.rank);
                s_fail = 1;
                break;
            }
            v = ptx::ld_acquire_sys_u64(f);
        }
        ps.wait_end();
        if (tokens_out) tokens_out[threadIdx.x] = static_cast<uint32_t>(v);
    }
    __syncthreads();
    return s_fail == 0;
}

// ---------------------------------------------------------------------------

__global__ void begin_kernel(EpConfig c, EpWorkspace ws) {
    PhaseScope ps_(ws.debug_time, kPhaseBegin);
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        *ws.epoch += 1;
        if (*reinterpret_cast<volatile uint32_t*>(ws.error) != 0) {
            // Errors persist until the owner clears them; never run a round on a poisoned workspace silently.
        }
    }
    for (int e = threadIdx.x; e < c.experts_per_rank; e += blockDim.x) {
        ws.expert_count[e] = 0;
        ws.cursor[e] = 0;
    }
}

template <int MAXV>
__global__ void __launch_bounds__(kThreads) route_kernel(const float* logits, int tokens, int experts, int topk,
                                                         int32_t* idx, float* w, uint64_t* dbg) {
    PhaseScope ps_(dbg, kPhaseRoute);
    const int lane = threadIdx.x & 31;
    const int t = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
    if (t >= tokens) return;
    const float* row = logits + static_cast<int64_t>(t) * experts;
    float v[MAXV];
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int j = lane + 32 * i;
        v[i] = j < experts ? row[j] : -INFINITY;
    }
    float top_v[kMaxTopk];
    int top_i[kMaxTopk];
#pragma unroll
    for (int r = 0; r < kMaxTopk; ++r) {
        if (r >= topk) break;
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < MAXV; ++i) {
            const int j = lane + 32 * i;
            if (v[i] > bv || (v[i] == bv && j < bi)) {
                bv = v[i];
                bi = j;
            }
        }
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, d);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, d);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        top_v[r] = bv;
        top_i[r] = bi;
#pragma unroll
        for (int i = 0; i < MAXV; ++i) {
            if (lane + 32 * i == bi) v[i] = -INFINITY;
        }
    }
    float sum = 0.f;
#pragma unroll
    for (int r = 0; r < kMaxTopk; ++r) {
        if (r < topk) sum += __expf(top_v[r] - top_v[0]);
    }
#pragma unroll
    for (int r = 0; r < kMaxTopk; ++r) {
        if (r < topk && lane == r) {
            idx[static_cast<int64_t>(t) * topk + r] = top_i[r];
            w[static_cast<int64_t>(t) * topk + r] = __expf(top_v[r] - top_v[0]) / sum;
        }
    }
}

/// Copies `bytes` (a multiple of 16) from this warp's shared staging to a
/// (possibly remote) slot, 16 bytes per lane per instruction.
KIWI_DEV void warp_copy_out(uint8_t* dst, const uint8_t* src, int bytes, int lane) {
    for (int o = lane * 16; o < bytes; o += 32 * 16) {
        ptx::st_v4(dst + o, *reinterpret_cast<const uint4*>(src + o));
    }
}

/// Dispatch: one warp per token.  The row is quantised 512 columns at a time
/// and each 16-byte lane chunk is stored straight into every destination
/// rank's receive slot over NVLink; the token's metadata (epoch, token, top-k
/// ids and weights) and its scales are first assembled in the warp's shared
/// staging in the slot's own layout and then stored with 16-byte vector
/// stores, so no destination sees a stream of 1- or 4-byte remote writes.
template <int QUANT>
__global__ void __launch_bounds__(kThreads) dispatch_kernel(EpConfig c, p2p::HeapView h, const __nv_bfloat16* x,
                                                            const int32_t* idx, const float* w, int tokens,
                                                            EpWorkspace ws, const uint8_t* raw_scales,
                                                            int raw_scale_bytes) {
    PhaseScope ps_(ws.debug_time, kPhaseDispatch);
    extern __shared__ __align__(16) uint8_t dyn_smem[];
    const int lane = threadIdx.x & 31;
    const int warp_in_block = threadIdx.x / 32;
    const int warps = gridDim.x * (blockDim.x / 32);
    const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(ws.epoch);
    const int me = c.rank;
    // Per-warp staging: [meta_bytes][scale_bytes], both 16-byte multiples.
    uint8_t* stage = dyn_smem + warp_in_block * (c.meta_bytes + c.scale_bytes);
    uint8_t* s_meta = stage;
    uint8_t* s_scale = stage + c.meta_bytes;
    for (int t = (blockIdx.x * blockDim.x + threadIdx.x) / 32; t < tokens; t += warps) {
        const int e = lane < c.topk ? idx[static_cast<int64_t>(t) * c.topk + lane] : -1;
        const float wt = lane < c.topk ? w[static_cast<int64_t>(t) * c.topk + lane] : 0.f;
        const bool ok_e = e >= 0 && e < c.num_experts;
        const uint32_t mask = __reduce_or_sync(0xffffffffu, ok_e ? (1u << (e / c.experts_per_rank)) : 0u);
        const uint64_t slot = c.slot_index(me, t);
        __syncwarp();  // the previous token's staging has been stored
        if (lane < c.topk) {
            reinterpret_cast<int32_t*>(s_meta + sizeof(DispatchMetaHeader))[lane] = e;
            reinterpret_cast<float*>(s_meta + sizeof(DispatchMetaHeader) + 4 * c.topk)[lane] = wt;
        }
        if (lane == 0) *reinterpret_cast<uint4*>(s_meta) = make_uint4(epoch, static_cast<uint32_t>(t), 0, 0);
        const int meta_pad_from = static_cast<int>(sizeof(DispatchMetaHeader)) + 8 * c.topk;
        for (int o = meta_pad_from + lane * 4; o < c.meta_bytes; o += 32 * 4) {
            *reinterpret_cast<uint32_t*>(s_meta + o) = 0;
        }
        const __nv_bfloat16* xr = x + static_cast<int64_t>(t) * c.hidden;
        if constexpr (QUANT == kDispatchRaw) {
            // Pre-quantised by the caller: the row's wire bytes travel unchanged.
            const uint8_t* rr = reinterpret_cast<const uint8_t*>(x) + static_cast<int64_t>(t) * c.row_bytes;
            for (int o = lane * 16; o < c.row_bytes; o += 32 * 16) {
                const uint4 v = ptx::ld_nc_v4(rr + o);
                for (uint32_t m = mask; m; m &= m - 1) {
                    const int r = __ffs(m) - 1;
                    ptx::st_v4(h.base[r] + c.row_off(slot) + o, v);
                }
            }
        } else if constexpr (QUANT == static_cast<int>(Quant::kNone)) {
            for (int col = lane * 8; col < c.hidden; col += 256) {
                const uint4 v = ptx::ld_nc_v4(xr + col);
                for (uint32_t m = mask; m; m &= m - 1) {
                    const int r = __ffs(m) - 1;
                    ptx::st_v4(h.base[r] + c.row_off(slot) + 2ull * col, v);
                }
            }
        } else if constexpr (QUANT == static_cast<int>(Quant::kFp8)) {
            for (int base = 0; base < c.hidden; base += 512) {
                const int col = base + lane * 16;
                uint4 in[2];
                in[0] = ptx::ld_nc_v4(xr + col);
                in[1] = ptx::ld_nc_v4(xr + col + 8);
                float scale;
                uint4 q;
                quant_fp8_16(in, scale, q);
                if ((lane & 7) == 0) reinterpret_cast<float*>(s_scale)[col / kFp8Block] = scale;
                for (uint32_t m = mask; m; m &= m - 1) {
                    const int r = __ffs(m) - 1;
                    ptx::st_v4(h.base[r] + c.row_off(slot) + col, q);
                }
            }
        } else {
            // NVFP4: per-row fp32 scale first (row amax / (448 * 6)), then 16-element blocks.
            float amax = 0.f;
            for (int col = lane * 8; col < c.hidden; col += 256) {
                float f[8];
                bf16x8_to_f32(ptx::ld_nc_v4(xr + col), f);
#pragma unroll
                for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(f[i]));
            }
#pragma unroll
            for (int d = 16; d > 0; d >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, d));
            const float row_scale = amax > 0.f ? amax / (kFp8Max * kFp4Max) : 0.f;
            if (lane == 0) reinterpret_cast<float*>(s_scale)[0] = row_scale;
            for (int base = 0; base < c.hidden; base += 512) {
                const int col = base + lane * 16;
                uint4 in[2];
                in[0] = ptx::ld_nc_v4(xr + col);
                in[1] = ptx::ld_nc_v4(xr + col + 8);
                uint8_t sb;
                uint2 q;
                quant_fp4_16(in, row_scale, sb, q);
                s_scale[4 + col / kFp4Block] = sb;
                for (uint32_t m = mask; m; m &= m - 1) {
                    const int r = __ffs(m) - 1;
                    *reinterpret_cast<uint2*>(h.base[r] + c.row_off(slot) + col / 2) = q;
                }
            }
            // Zero the staging tail past the last block scale (the slot layout pads to 16 bytes).
            for (int o = 4 + c.hidden / kFp4Block + lane; o < c.scale_bytes; o += 32) s_scale[o] = 0;
        }
        if (raw_scales) {
            // The caller's own per-token scales (bf16 or pre-quantised rows): copied
            // as bytes, zero padded to the slot's scale room.
            const uint8_t* sr = raw_scales + static_cast<int64_t>(t) * raw_scale_bytes;
            for (int o = lane; o < c.scale_bytes; o += 32) s_scale[o] = o < raw_scale_bytes ? sr[o] : 0;
        }
        __syncwarp();
        for (uint32_t m = mask; m; m &= m - 1) {
            const int r = __ffs(m) - 1;
            warp_copy_out(h.base[r] + c.meta_off(slot), s_meta, c.meta_bytes, lane);
            if (c.scale_bytes) warp_copy_out(h.base[r] + c.scale_off(slot), s_scale, c.scale_bytes, lane);
        }
    }
    grid_done_signal(c, h, &ws.done_ctas[0], c.dispatch_flag(me),
                     (static_cast<uint64_t>(epoch) << 32) | static_cast<uint32_t>(tokens));
}

/// One warp waits for every rank's dispatch (which == 0) or combine
/// (which == 1) flag of this round and, for dispatch, records each source's
/// token count in ws.slot_tokens.  Launched on its own ahead of the kernel
/// that reads the data (which is then launched with waited = true), so the
/// only kernel that spins on another GPU is this 32-thread one: it never
/// holds the SMs that a concurrently scheduled kernel of another stream needs.
__global__ void __launch_bounds__(32) wait_flags_kernel(EpConfig c, p2p::HeapView h, EpWorkspace ws, int which,
                                                        uint64_t timeout_ns) {
    PhaseScope ps_(ws.debug_time, which == 0 ? kPhaseDispatchWait : kPhaseCombineWait);
    __shared__ uint32_t s_tokens[kMaxRanks];
    const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(ws.epoch);
    const bool ok = which == 0
                        ? wait_all_flags(c, h, ws, epoch, [&](int src) { return c.dispatch_flag(src); },
                                         kSiteDispatchWait, timeout_ns, s_tokens, ps_)
                        : wait_all_flags(c, h, ws, epoch, [&](int src) { return c.combine_flag(src); },
                                         kSiteCombineWait, timeout_ns, nullptr, ps_);
    if (ok && which == 0 && threadIdx.x < static_cast<unsigned>(c.world)) ws.slot_tokens[threadIdx.x] = s_tokens[threadIdx.x];
}

/// True when an earlier kernel of this round recorded an error (a wait ran out).
KIWI_DEV bool round_failed(const EpWorkspace& ws) { return *reinterpret_cast<volatile uint32_t*>(ws.error) != 0; }

__global__ void __launch_bounds__(kThreads) recv_count_kernel(EpConfig c, p2p::HeapView h, EpWorkspace ws,
                                                              uint64_t timeout_ns, int waited) {
    PhaseScope ps_(ws.debug_time, kPhaseRecvCount);
    __shared__ uint32_t s_tokens[kMaxRanks];
    const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(ws.epoch);
    if (waited) {
        // wait_flags_kernel ran first on this stream and stored the counts.
        if (round_failed(ws)) return;
        if (threadIdx.x < static_cast<unsigned>(c.world)) {
            s_tokens[threadIdx.x] = static_cast<uint32_t>(*reinterpret_cast<volatile int32_t*>(ws.slot_tokens + threadIdx.x));
        }
        __syncthreads();
    } else {
        if (!wait_all_flags(c, h, ws, epoch, [&](int src) { return c.dispatch_flag(src); }, kSiteDispatchWait,
                            timeout_ns, s_tokens, ps_)) {
            return;
        }
        if (blockIdx.x == 0 && threadIdx.x < static_cast<unsigned>(c.world)) ws.slot_tokens[threadIdx.x] = s_tokens[threadIdx.x];
    }
    const int e0 = c.rank * c.experts_per_rank;
    const uint8_t* base = h.base[h.rank];
    for (uint64_t s = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; s < c.slots();
         s += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const int src = static_cast<int>(s / c.max_tokens);
        const int t = static_cast<int>(s % c.max_tokens);
        if (t >= static_cast<int>(s_tokens[src])) continue;
        const uint8_t* mp = meta_ptr(c, base, s);
        if (ld_cg_u32(mp) != epoch) continue;
        const int32_t* ids = reinterpret_cast<const int32_t*>(mp + sizeof(DispatchMetaHeader));
        for (int j = 0; j < c.topk; ++j) {
            const int e = static_cast<int>(ld_cg_u32(ids + j)) - e0;
            if (e >= 0 && e < c.experts_per_rank) atomicAdd(&ws.expert_count[e], 1);
        }
    }
}

/// Receive, step 1 (warp per slot): validates the slot, assigns one
/// expert-major row per local expert with an atomic per expert, and records
/// pair_slot / pair_w and the slot's row list (slot_pos, -1 padded).
__global__ void __launch_bounds__(kThreads) recv_assign_kernel(EpConfig c, p2p::HeapView h, EpWorkspace ws) {
    PhaseScope ps_(ws.debug_time, kPhaseRecvAssign);
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (blockDim.x / 32);
    const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(ws.epoch);
    const int e0 = c.rank * c.experts_per_rank;
    const int lpt = c.local_per_token();
    const uint8_t* base = h.base[h.rank];
    const int64_t max_pairs = c.max_pairs();
    for (uint64_t s = (blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x) / 32; s < c.slots();
         s += warps) {
        const int src = static_cast<int>(s / c.max_tokens);
        const int t = static_cast<int>(s % c.max_tokens);
        const uint8_t* mp = meta_ptr(c, base, s);
        bool valid = t < ws.slot_tokens[src];
        if (valid) valid = ld_cg_u32(mp) == epoch;
        int e = -1;
        float wt = 0.f;
        if (valid && lane < c.topk) {
            e = static_cast<int>(ld_cg_u32(reinterpret_cast<const int32_t*>(mp + sizeof(DispatchMetaHeader)) + lane)) - e0;
            wt = ld_cg_f32(reinterpret_cast<const float*>(mp + sizeof(DispatchMetaHeader) + 4 * c.topk) + lane);
        }
        const bool local = valid && lane < c.topk && e >= 0 && e < c.experts_per_rank;
        const uint32_t lmask = __ballot_sync(0xffffffffu, local);
        if (local) {
            int pos = ws.offsets[e] + atomicAdd(&ws.cursor[e], 1);
            if (pos < max_pairs) {
                ws.pair_slot[pos] = static_cast<int32_t>(s);
                ws.pair_w[pos] = wt;
                if (ws.pair_dst) {
                    ws.pair_dst[pos] = (static_cast<int64_t>(src) << 48) | static_cast<int64_t>(c.combk_off(t, lane));
                }
            } else {
                set_error(ws, static_cast<uint32_t>(Status::kBadArgument), kSiteCapacity, pos, c.rank);
                pos = -1;
            }
            const int r = __popc(lmask & ((1u << lane) - 1));
            if (r < lpt) {
                ws.slot_pos[s * lpt + r] = pos;
            } else {
                // More local experts than local_per_token: only possible with
                // repeated expert ids in caller-supplied routing.
                set_error(ws, static_cast<uint32_t>(Status::kBadArgument), kSiteCapacity, r, c.rank);
            }
        }
        const int nloc = __popc(lmask);
        if (lane >= nloc && lane < lpt) ws.slot_pos[s * lpt + lane] = -1;
    }
}

/// Raw bytes of one receive item (a slot's 512-column block) as loaded.
struct RecvRaw {
    uint4 q0, q1;
    float s0;
    uint32_t s1;
};

template <int QUANT>
KIWI_DEV void recv_load(const EpConfig& c, const uint8_t* base, uint64_t s, int col, int lane, RecvRaw& r) {
    if constexpr (QUANT == static_cast<int>(Quant::kNone)) {
        r.q0 = ld_cg_v4(base + c.row_off(s) + 2ull * col);
        r.q1 = ld_cg_v4(base + c.row_off(s) + 2ull * col + 16);
    } else if constexpr (QUANT == static_cast<int>(Quant::kFp8)) {
        r.q0 = ld_cg_v4(base + c.row_off(s) + col);
        r.s0 = ld_cg_f32(base + c.scale_off(s) + 4ull * (col / kFp8Block));
    } else {
        r.q0 = ld_cg_v4(base + c.row_off(s) + (col / 32) * 16);  // 16 B = 32 elements (a lane pair)
        r.s0 = ld_cg_f32(base + c.scale_off(s));
        r.s1 = ld_cg_u32(base + c.scale_off(s) + 4 + ((col / kFp4Block) & ~3));
    }
}

template <int QUANT>
KIWI_DEV void recv_convert(int col, int lane, const RecvRaw& r, uint4 (&out)[2]) {
    if constexpr (QUANT == static_cast<int>(Quant::kNone)) {
        out[0] = r.q0;
        out[1] = r.q1;
    } else if constexpr (QUANT == static_cast<int>(Quant::kFp8)) {
        dequant_fp8_16(r.q0, r.s0, out);
    } else {
        const uint2 q = (lane & 1) ? make_uint2(r.q0.z, r.q0.w) : make_uint2(r.q0.x, r.q0.y);
        const uint8_t sb = static_cast<uint8_t>(r.s1 >> (8 * ((col / kFp4Block) & 3)));
        const __half_raw sh = __nv_cvt_fp8_to_halfraw(sb, __NV_E4M3);
        dequant_fp4_16(q, __half2float(*reinterpret_cast<const __half*>(&sh)) * r.s0, out);
    }
}

/// Receive, step 2: for every (valid slot, 512-column block) the warp loads the
/// dispatched bytes once, dequantises them and stores the bf16 row block into
/// each of the slot's expert-major rows.  Items are spread over the whole grid
/// and each warp keeps two items' loads in flight (the kernel is load-latency
/// bound: ncu showed long-scoreboard stalls dominating at 79 % warp occupancy).
template <int QUANT>
__global__ void __launch_bounds__(kThreads) recv_copy_kernel(EpConfig c, p2p::HeapView h, EpWorkspace ws) {
    PhaseScope ps_(ws.debug_time, kPhaseRecvCopy);
    const int lane = threadIdx.x & 31;
    const uint64_t warps = gridDim.x * (blockDim.x / 32);
    const int lpt = c.local_per_token();
    const uint8_t* base = h.base[h.rank];
    const int blocks = c.hidden / 512;
    const uint64_t items = c.slots() * blocks;
    for (uint64_t it = (blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x) / 32; it < items;
         it += 2 * warps) {
        uint64_t s[2];
        int col[2], p[2];
        uint32_t pm[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const uint64_t i = it + u * warps;
            s[u] = i / blocks;
            col[u] = static_cast<int>(i % blocks) * 512 + lane * 16;
            p[u] = (i < items && lane < lpt) ? ws.slot_pos[s[u] * lpt + lane] : -1;
        }
        RecvRaw raw[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            pm[u] = __ballot_sync(0xffffffffu, p[u] >= 0);
            if (pm[u]) recv_load<QUANT>(c, base, s[u], col[u], lane, raw[u]);
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            if (pm[u] == 0) continue;
            uint4 out[2];
            recv_convert<QUANT>(col[u], lane, raw[u], out);
            for (uint32_t m = pm[u]; m; m &= m - 1) {
                const int pp = __shfl_sync(0xffffffffu, p[u], __ffs(m) - 1);
                __nv_bfloat16* dst = ws.a + static_cast<int64_t>(pp) * c.hidden + col[u];
                ptx::st_v4(dst, out[0]);
                ptx::st_v4(dst + 8, out[1]);
            }
        }
    }
}

/// Sums up to MAXP bf16 rows (load(j) for j < n) into fp32: every load is
/// issued before the first add so all of them are in flight together.
template <int MAXP, typename Loader>
KIWI_DEV void sum_rows(int n, Loader load, float (&acc)[8]) {
    uint4 v[MAXP];
#pragma unroll
    for (int j = 0; j < MAXP; ++j) {
        if (j < n) v[j] = load(j);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll
    for (int j = 0; j < MAXP; ++j) {
        if (j < n) {
            float f[8];
            bf16x8_to_f32(v[j], f);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] += f[i];
        }
    }
}

/// Combine, send side: for every (slot, 256-column block) the warp sums the
/// slot's (already routing-weighted) expert rows and stores the bf16 block into
/// the token owner's combine slot over NVLink.  MAXP bounds the rows per slot.
template <int MAXP>
__global__ void __launch_bounds__(kThreads) combine_send_kernel(EpConfig c, p2p::HeapView h,
                                                                const __nv_bfloat16* y, EpWorkspace ws) {
    PhaseScope ps_(ws.debug_time, kPhaseCombineSend);
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (blockDim.x / 32);
    const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(ws.epoch);
    const int lpt = c.local_per_token();
    const int blocks = c.hidden / 256;
    const uint64_t items = c.slots() * blocks;
    for (uint64_t it = (blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x) / 32; it < items; it += warps) {
        const uint64_t s = it / blocks;
        const int col = static_cast<int>(it % blocks) * 256 + lane * 8;
        const int p = lane < lpt ? ws.slot_pos[s * lpt + lane] : -1;
        const uint32_t pm = __ballot_sync(0xffffffffu, p >= 0);
        if (pm == 0) continue;
        const int npos = __popc(pm);  // positions are packed at the front of the slot's list
        int pl[MAXP];
#pragma unroll
        for (int j = 0; j < MAXP; ++j) pl[j] = __shfl_sync(0xffffffffu, p, j);
        const int src = static_cast<int>(s / c.max_tokens);
        const int t = static_cast<int>(s % c.max_tokens);
        float acc[8];
        sum_rows<MAXP>(npos, [&](int j) { return ptx::ld_v4(y + static_cast<int64_t>(pl[j]) * c.hidden + col); }, acc);
        ptx::st_v4(h.base[src] + c.comb_off(c.rank, t) + 2ull * col, f32x8_to_bf16(acc));
    }
    grid_done_signal(c, h, &ws.done_ctas[1], c.combine_flag(c.rank), (static_cast<uint64_t>(epoch) << 32) | 1u);
}

/// Raw bytes of 8 consecutive elements of a combine row in CombDtype DT
/// (bf16: 16 bytes, fp32: 32, FP8: 8, FP4: 4).
struct Comb8 {
    uint4 a, b;
};

template <int DT>
KIWI_DEV Comb8 comb_load8(const uint8_t* row, int col) {
    Comb8 r{make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
    if constexpr (DT == static_cast<int>(CombDtype::kBf16)) {
        r.a = ld_cg_v4(row + 2ull * col);
    } else if constexpr (DT == static_cast<int>(CombDtype::kF32)) {
        r.a = ld_cg_v4(row + 4ull * col);
        r.b = ld_cg_v4(row + 4ull * col + 16);
    } else if constexpr (DT == static_cast<int>(CombDtype::kFp8)) {
        const uint2 v = ld_cg_v2(row + col);
        r.a.x = v.x;
        r.a.y = v.y;
    } else {
        r.a.x = ld_cg_u32(row + col / 2);
    }
    return r;
}

template <int DT>
KIWI_DEV void comb_decode8(const Comb8& r, float (&f)[8]) {
    if constexpr (DT == static_cast<int>(CombDtype::kBf16)) {
        bf16x8_to_f32(r.a, f);
    } else if constexpr (DT == static_cast<int>(CombDtype::kF32)) {
        f[0] = __uint_as_float(r.a.x); f[1] = __uint_as_float(r.a.y);
        f[2] = __uint_as_float(r.a.z); f[3] = __uint_as_float(r.a.w);
        f[4] = __uint_as_float(r.b.x); f[5] = __uint_as_float(r.b.y);
        f[6] = __uint_as_float(r.b.z); f[7] = __uint_as_float(r.b.w);
    } else if constexpr (DT == static_cast<int>(CombDtype::kFp8)) {
        const uint32_t w[2] = {r.a.x, r.a.y};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(
                static_cast<__nv_fp8x2_storage_t>((w[i / 2] >> (16 * (i & 1))) & 0xffffu), __NV_E4M3);
            const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&hr));
            f[2 * i] = t.x;
            f[2 * i + 1] = t.y;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const __half2_raw hr =
                __nv_cvt_fp4x2_to_halfraw2(static_cast<__nv_fp4x2_storage_t>((r.a.x >> (8 * i)) & 0xffu), __NV_E2M1);
            const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&hr));
            f[2 * i] = t.x;
            f[2 * i + 1] = t.y;
        }
    }
}

/// Stores 8 fp32 values as combine-row elements of CombDtype DT; FP8 and FP4
/// round to nearest and saturate (e4m3 at +-448, e2m1 at +-6).
template <int DT>
KIWI_DEV void comb_store8(uint8_t* row, int col, const float (&f)[8]) {
    if constexpr (DT == static_cast<int>(CombDtype::kBf16)) {
        ptx::st_v4(row + 2ull * col, f32x8_to_bf16(f));
    } else if constexpr (DT == static_cast<int>(CombDtype::kF32)) {
        ptx::st_v4(row + 4ull * col, make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                                                 __float_as_uint(f[3])));
        ptx::st_v4(row + 4ull * col + 16, make_uint4(__float_as_uint(f[4]), __float_as_uint(f[5]),
                                                      __float_as_uint(f[6]), __float_as_uint(f[7])));
    } else if constexpr (DT == static_cast<int>(CombDtype::kFp8)) {
        uint32_t w[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(f[4 * i], f[4 * i + 1]), __NV_SATFINITE, __NV_E4M3);
            const uint32_t hi =
                __nv_cvt_float2_to_fp8x2(make_float2(f[4 * i + 2], f[4 * i + 3]), __NV_SATFINITE, __NV_E4M3);
            w[i] = lo | (hi << 16);
        }
        *reinterpret_cast<uint2*>(row + col) = make_uint2(w[0], w[1]);
    } else {
        uint32_t w = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            w |= static_cast<uint32_t>(__nv_cvt_float2_to_fp4x2(make_float2(f[2 * i], f[2 * i + 1]), __NV_E2M1,
                                                                 cudaRoundNearest))
                 << (8 * i);
        }
        *reinterpret_cast<uint32_t*>(row + col / 2) = w;
    }
}

/// Combine, receive side: after every rank's flag, each (token, 256-column
/// block) sums, in fp32, the rows the token's destination ranks returned and
/// writes the sum in the combine dtype DT.  With out_w, the (token, block 0)
/// item also sums the top-k weights that came back with those rows.
template <int DT, int MAXR>
__global__ void __launch_bounds__(kThreads) combine_recv_kernel(EpConfig c, p2p::HeapView h, const int32_t* idx,
                                                                int tokens, uint8_t* out, float* out_w,
                                                                EpWorkspace ws, uint64_t timeout_ns, int waited) {
    PhaseScope ps_(ws.debug_time, kPhaseCombineRecv);
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (blockDim.x / 32);
    const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(ws.epoch);
    if (waited) {
        if (round_failed(ws)) return;
    } else if (!wait_all_flags(c, h, ws, epoch, [&](int src) { return c.combine_flag(src); }, kSiteCombineWait,
                               timeout_ns, nullptr, ps_)) {
        return;
    }
    const uint8_t* base = h.base[h.rank];
    const int blocks = (c.hidden + 255) / 256;
    const uint64_t items = static_cast<uint64_t>(tokens) * blocks;
    for (uint64_t it = (blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x) / 32; it < items; it += warps) {
        const int t = static_cast<int>(it / blocks);
        const int blk = static_cast<int>(it % blocks);
        const int col = blk * 256 + lane * 8;
        const int e = lane < c.topk ? idx[static_cast<int64_t>(t) * c.topk + lane] : -1;
        const bool ok_e = e >= 0 && e < c.num_experts;
        uint32_t m = __reduce_or_sync(0xffffffffu, ok_e ? (1u << (e / c.experts_per_rank)) : 0u);
        int rl[MAXR];
        int nr = 0;
#pragma unroll
        for (int j = 0; j < MAXR; ++j) {
            rl[j] = m ? __ffs(m) - 1 : 0;
            if (m) {
                ++nr;
                m &= m - 1;
            }
        }
        if (col < c.hidden) {
            Comb8 v[MAXR];
#pragma unroll
            for (int j = 0; j < MAXR; ++j) {
                if (j < nr) v[j] = comb_load8<DT>(base + c.comb_off(rl[j], t), col);
            }
            float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int j = 0; j < MAXR; ++j) {
                if (j < nr) {
                    float f[8];
                    comb_decode8<DT>(v[j], f);
#pragma unroll
                    for (int i = 0; i < 8; ++i) acc[i] += f[i];
                }
            }
            comb_store8<DT>(out + static_cast<int64_t>(t) * c.comb_row_bytes, col, acc);
        }
        if (out_w && blk == 0 && lane < c.topk) {
            float sw = 0.f;
            for (int j = 0; j < nr; ++j) {
                sw += ld_cg_f32(base + c.comb_off(rl[j], t) + c.comb_row_bytes + 4 * lane);
            }
            out_w[static_cast<int64_t>(t) * c.topk + lane] = sw;
        }
    }
}

/// Fused combine, receive side: (token, 256-column block) items sum the
/// token's top-k combk rows (each written by the rank owning that expert).
template <int MAXK>
__global__ void __launch_bounds__(kThreads) combine_recv_fused_kernel(EpConfig c, p2p::HeapView h, const int32_t* idx,
                                                                      int tokens, __nv_bfloat16* out, EpWorkspace ws,
                                                                      uint64_t timeout_ns, int waited) {
    PhaseScope ps_(ws.debug_time, kPhaseCombineRecv);
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (blockDim.x / 32);
    const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(ws.epoch);
    if (waited) {
        if (round_failed(ws)) return;
    } else if (!wait_all_flags(c, h, ws, epoch, [&](int src) { return c.combine_flag(src); }, kSiteCombineWait,
                               timeout_ns, nullptr, ps_)) {
        return;
    }
    const uint8_t* base = h.base[h.rank];
    const int blocks = c.hidden / 256;
    const uint64_t items = static_cast<uint64_t>(tokens) * blocks;
    for (uint64_t it = (blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x) / 32; it < items; it += warps) {
        const int t = static_cast<int>(it / blocks);
        const int col = static_cast<int>(it % blocks) * 256 + lane * 8;
        const int e = lane < c.topk ? idx[static_cast<int64_t>(t) * c.topk + lane] : -1;
        uint32_t m = __ballot_sync(0xffffffffu, e >= 0 && e < c.num_experts);
        int kl[MAXK];
        int nk = 0;
#pragma unroll
        for (int j = 0; j < MAXK; ++j) {
            kl[j] = m ? __ffs(m) - 1 : 0;
            if (m) {
                ++nk;
                m &= m - 1;
            }
        }
        float acc[8];
        sum_rows<MAXK>(nk, [&](int j) { return ld_cg_v4(base + c.combk_off(t, kl[j]) + 2ull * col); }, acc);
        ptx::st_v4(out + static_cast<int64_t>(t) * c.hidden + col, f32x8_to_bf16(acc));
    }
}


// ---------------------------------------------------------------------------
// Transport-only path (rows in, rows out), MORI semantics.
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(1024) recv_compact_kernel(EpConfig c, p2p::HeapView h, EpWorkspace ws,
                                                            int32_t* slot_compact, int32_t* recv_count) {
    PhaseScope ps_(ws.debug_time, kPhaseRecvCompact);
    __shared__ int32_t s_scan[1024];
    __shared__ int32_t s_base;
    const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(ws.epoch);
    const uint8_t* base = h.base[h.rank];
    if (threadIdx.x == 0) s_base = 0;
    __syncthreads();
    for (uint64_t s0 = 0; s0 < c.slots(); s0 += blockDim.x) {
        const uint64_t s = s0 + threadIdx.x;
        int valid = 0;
        if (s < c.slots()) {
            const int src = static_cast<int>(s / c.max_tokens);
            const int t = static_cast<int>(s % c.max_tokens);
            valid = (t < ws.slot_tokens[src] && ld_cg_u32(meta_ptr(c, base, s)) == epoch) ? 1 : 0;
        }
        s_scan[threadIdx.x] = valid;
        __syncthreads();
        for (int d = 1; d < blockDim.x; d <<= 1) {
            const int v = threadIdx.x >= static_cast<unsigned>(d) ? s_scan[threadIdx.x - d] : 0;
            __syncthreads();
            s_scan[threadIdx.x] += v;
            __syncthreads();
        }
        if (s < c.slots()) slot_compact[s] = valid ? s_base + s_scan[threadIdx.x] - 1 : -1;
        __syncthreads();
        if (threadIdx.x == blockDim.x - 1) s_base += s_scan[threadIdx.x];
        __syncthreads();
    }
    if (threadIdx.x == 0) *recv_count = s_base;
}

__global__ void __launch_bounds__(kThreads) gather_rows_kernel(EpConfig c, p2p::HeapView h, EpWorkspace ws,
                                                               const int32_t* slot_compact, uint8_t* out_rows,
                                                               uint8_t* out_scales, int32_t* out_idx, float* out_w,
                                                               int32_t* out_src_pos) {
    PhaseScope ps_(ws.debug_time, kPhaseGatherRows);
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (blockDim.x / 32);
    const uint8_t* base = h.base[h.rank];
    for (uint64_t s = (blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x) / 32; s < c.slots();
         s += warps) {
        const int pos = slot_compact[s];
        if (pos < 0) continue;
        const uint8_t* mp = meta_ptr(c, base, s);
        if (lane < c.topk) {
            out_idx[static_cast<int64_t>(pos) * c.topk + lane] =
                static_cast<int32_t>(ld_cg_u32(mp + sizeof(DispatchMetaHeader) + 4 * lane));
            out_w[static_cast<int64_t>(pos) * c.topk + lane] =
                ld_cg_f32(mp + sizeof(DispatchMetaHeader) + 4 * c.topk + 4 * lane);
        }
        if (lane == 0) out_src_pos[pos] = static_cast<int32_t>(s);
        const uint8_t* row = base + c.row_off(s);
        uint8_t* dst = out_rows + static_cast<int64_t>(pos) * c.row_bytes;
        for (int off = lane * 16; off < c.row_bytes; off += 512) ptx::st_v4(dst + off, ld_cg_v4(row + off));
        if (c.scale_bytes) {
            const uint8_t* sc = base + c.scale_off(s);
            uint8_t* sd = out_scales + static_cast<int64_t>(pos) * c.scale_bytes;
            for (int off = lane * 16; off < c.scale_bytes; off += 512) ptx::st_v4(sd + off, ld_cg_v4(sc + off));
        }
    }
}

__global__ void __launch_bounds__(kThreads) combine_rows_kernel(EpConfig c, p2p::HeapView h, const uint8_t* rows,
                                                                const float* weights, const int32_t* src_pos,
                                                                const int32_t* recv_count, EpWorkspace ws) {
    PhaseScope ps_(ws.debug_time, kPhaseCombineRows);
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (blockDim.x / 32);
    const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(ws.epoch);
    const int n = *recv_count;
    for (int i = (blockIdx.x * blockDim.x + threadIdx.x) / 32; i < n; i += warps) {
        const int sp = src_pos[i];
        const int src = sp / c.max_tokens;
        const int t = sp % c.max_tokens;
        uint8_t* dst = h.base[src] + c.comb_off(c.rank, t);
        const uint8_t* r = rows + static_cast<int64_t>(i) * c.comb_row_bytes;
        for (int o = lane * 16; o < c.comb_row_bytes; o += 32 * 16) ptx::st_v4(dst + o, ptx::ld_v4(r + o));
        if (weights && c.comb_weights && lane < c.topk) {
            *reinterpret_cast<float*>(dst + c.comb_row_bytes + 4 * lane) =
                weights[static_cast<int64_t>(i) * c.topk + lane];
        }
    }
    grid_done_signal(c, h, &ws.done_ctas[1], c.combine_flag(c.rank), (static_cast<uint64_t>(epoch) << 32) | 1u);
}

/// SM count of the current device (cached per device: a process may drive several GPUs).
int default_grid() {
    static std::atomic<int> cached[64] = {};
    int dev = 0;
    KIWI_CUDA_CHECK(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) throw kiwi::error("kiwi::ep: device index beyond 64");
    int n = cached[dev].load(std::memory_order_relaxed);
    if (n == 0) {
        KIWI_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
        cached[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

}  // namespace

void launch_begin(const EpConfig& c, const EpWorkspace& ws, cudaStream_t s) {
    begin_kernel<<<1, 256, 0, s>>>(c, ws);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

void launch_route(const float* logits, int tokens, int experts, int topk, int32_t* idx, float* w, cudaStream_t s,
                  uint64_t* debug_time) {
    if (topk < 1 || topk > kMaxTopk) throw kiwi::error("route: topk must be in [1, 16]");
    if (tokens == 0) return;
    const int blocks = (tokens * 32 + kThreads - 1) / kThreads;
    if (experts <= 64) route_kernel<2><<<blocks, kThreads, 0, s>>>(logits, tokens, experts, topk, idx, w, debug_time);
    else if (experts <= 256) route_kernel<8><<<blocks, kThreads, 0, s>>>(logits, tokens, experts, topk, idx, w, debug_time);
    else if (experts <= 1024) route_kernel<32><<<blocks, kThreads, 0, s>>>(logits, tokens, experts, topk, idx, w, debug_time);
    else throw kiwi::error("route: at most 1024 experts");
    KIWI_CUDA_CHECK(cudaGetLastError());
}

int dispatch_grid(int tokens, int tuned, int sms) {
    if (tuned > 0) return tuned;
    // One warp per token up to 8 blocks per SM: dispatch is load- and
    // store-latency bound, so every token's loads should be in flight at once.
    const int want = (tokens * 32 + kThreads - 1) / kThreads;
    return std::max(1, std::min(want, 8 * std::max(1, sms)));
}

void launch_dispatch(const EpConfig& c, const p2p::HeapView& h, const __nv_bfloat16* x, const int32_t* idx,
                     const float* w, int tokens, const EpWorkspace& ws, int grid, cudaStream_t s,
                     const void* raw_scales, int raw_scale_bytes) {
    if (tokens > c.max_tokens) throw kiwi::error("dispatch: more tokens than max_tokens");
    if (raw_scales && (raw_scale_bytes <= 0 || raw_scale_bytes > c.scale_bytes)) {
        throw kiwi::error("dispatch: caller scales need 1..scale_bytes bytes per token");
    }
    if (raw_scales && c.quant != static_cast<int>(Quant::kNone)) {
        throw kiwi::error("dispatch: an FP8 / NVFP4 op makes its own scales from bf16 rows (use launch_dispatch_raw)");
    }
    grid = dispatch_grid(tokens, grid, default_grid());
    const size_t smem = static_cast<size_t>(kThreads / 32) * (c.meta_bytes + c.scale_bytes);
    if (smem > 48 * 1024) throw kiwi::error("dispatch: per-token staging exceeds 48 KB per block (hidden too large)");
    const uint8_t* rs = static_cast<const uint8_t*>(raw_scales);
    switch (static_cast<Quant>(c.quant)) {
        case Quant::kNone:
            dispatch_kernel<0><<<grid, kThreads, smem, s>>>(c, h, x, idx, w, tokens, ws, rs, raw_scale_bytes);
            break;
        case Quant::kFp8:
            dispatch_kernel<1><<<grid, kThreads, smem, s>>>(c, h, x, idx, w, tokens, ws, nullptr, 0);
            break;
        case Quant::kNvfp4:
            dispatch_kernel<2><<<grid, kThreads, smem, s>>>(c, h, x, idx, w, tokens, ws, nullptr, 0);
            break;
    }
    KIWI_CUDA_CHECK(cudaGetLastError());
}

void launch_dispatch_raw(const EpConfig& c, const p2p::HeapView& h, const void* rows, const void* scales,
                         int scale_row_bytes, const int32_t* idx, const float* w, int tokens, const EpWorkspace& ws,
                         int grid, cudaStream_t s) {
    if (tokens > c.max_tokens) throw kiwi::error("dispatch_raw: more tokens than max_tokens");
    if (c.quant == static_cast<int>(Quant::kNone)) throw kiwi::error("dispatch_raw: needs an FP8 or NVFP4 op");
    if (c.row_bytes % 16 != 0 || (reinterpret_cast<uintptr_t>(rows) & 15u) != 0) {
        throw kiwi::error("dispatch_raw: rows must be 16-byte aligned with a 16-byte multiple per row");
    }
    if (scales && (scale_row_bytes <= 0 || scale_row_bytes > c.scale_bytes)) {
        throw kiwi::error("dispatch_raw: caller scales need 1..scale_bytes bytes per token");
    }
    grid = dispatch_grid(tokens, grid, default_grid());
    const size_t smem = static_cast<size_t>(kThreads / 32) * (c.meta_bytes + c.scale_bytes);
    if (smem > 48 * 1024) throw kiwi::error("dispatch: per-token staging exceeds 48 KB per block (hidden too large)");
    dispatch_kernel<kDispatchRaw><<<grid, kThreads, smem, s>>>(c, h, static_cast<const __nv_bfloat16*>(rows), idx, w,
                                                               tokens, ws, static_cast<const uint8_t*>(scales),
                                                               scales ? scale_row_bytes : 0);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

void launch_wait_flags(const EpConfig& c, const p2p::HeapView& h, const EpWorkspace& ws, int which,
                       uint64_t timeout_ns, cudaStream_t s) {
    if (which != 0 && which != 1) throw kiwi::error("wait_flags: which is 0 (dispatch) or 1 (combine)");
    wait_flags_kernel<<<1, 32, 0, s>>>(c, h, ws, which, timeout_ns);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

void launch_recv_count(const EpConfig& c, const p2p::HeapView& h, const EpWorkspace& ws, uint64_t timeout_ns,
                       cudaStream_t s, bool waited) {
    const uint64_t blocks = (c.slots() + kThreads - 1) / kThreads;
    const int grid = static_cast<int>(blocks < 4u * default_grid() ? blocks : 4u * default_grid());
    recv_count_kernel<<<grid, kThreads, 0, s>>>(c, h, ws, timeout_ns, waited ? 1 : 0);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

void launch_recv_assign(const EpConfig& c, const p2p::HeapView& h, const EpWorkspace& ws, cudaStream_t s, int grid) {
    const uint64_t assign_blocks = (c.slots() * 32 + kThreads - 1) / kThreads;
    const uint64_t cap = grid > 0 ? static_cast<uint64_t>(grid) : 8u * default_grid();
    recv_assign_kernel<<<static_cast<int>(assign_blocks < cap ? assign_blocks : cap), kThreads, 0, s>>>(c, h, ws);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

void launch_recv_copy(const EpConfig& c, const p2p::HeapView& h, const EpWorkspace& ws, cudaStream_t s, int grid) {
    if (grid <= 0) grid = 8 * default_grid();
    switch (static_cast<Quant>(c.quant)) {
        case Quant::kNone: recv_copy_kernel<0><<<grid, kThreads, 0, s>>>(c, h, ws); break;
        case Quant::kFp8: recv_copy_kernel<1><<<grid, kThreads, 0, s>>>(c, h, ws); break;
        case Quant::kNvfp4: recv_copy_kernel<2><<<grid, kThreads, 0, s>>>(c, h, ws); break;
    }
    KIWI_CUDA_CHECK(cudaGetLastError());
}

void launch_recv_scatter(const EpConfig& c, const p2p::HeapView& h, const EpWorkspace& ws, cudaStream_t s) {
    launch_recv_assign(c, h, ws, s, 0);
    launch_recv_copy(c, h, ws, s, 0);
}

void launch_combine_send(const EpConfig& c, const p2p::HeapView& h, const __nv_bfloat16* y, const EpWorkspace& ws,
                         int grid, cudaStream_t s) {
    if (grid <= 0) grid = 8 * default_grid();
    if (c.local_per_token() <= 8) combine_send_kernel<8><<<grid, kThreads, 0, s>>>(c, h, y, ws);
    else combine_send_kernel<kMaxTopk><<<grid, kThreads, 0, s>>>(c, h, y, ws);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

void launch_combine_recv_fused(const EpConfig& c, const p2p::HeapView& h, const int32_t* idx, int tokens,
                               __nv_bfloat16* out, const EpWorkspace& ws, uint64_t timeout_ns, cudaStream_t s,
                               int grid, bool waited) {
    if (grid <= 0) grid = 8 * default_grid();
    const int wt = waited ? 1 : 0;
    if (c.topk <= 8) {
        combine_recv_fused_kernel<8><<<grid, kThreads, 0, s>>>(c, h, idx, tokens, out, ws, timeout_ns, wt);
    } else {
        combine_recv_fused_kernel<kMaxTopk><<<grid, kThreads, 0, s>>>(c, h, idx, tokens, out, ws, timeout_ns, wt);
    }
    KIWI_CUDA_CHECK(cudaGetLastError());
}

namespace {

template <int DT>
void launch_combine_recv_dt(const EpConfig& c, const p2p::HeapView& h, const int32_t* idx, int tokens, uint8_t* out,
                            float* out_w, const EpWorkspace& ws, uint64_t timeout_ns, cudaStream_t s, int grid,
                            int waited) {
    // A token's rows come from at most min(world, topk) ranks.
    if (c.world <= 8 || c.topk <= 8) {
        combine_recv_kernel<DT, 8><<<grid, kThreads, 0, s>>>(c, h, idx, tokens, out, out_w, ws, timeout_ns, waited);
    } else {
        combine_recv_kernel<DT, kMaxTopk>
            <<<grid, kThreads, 0, s>>>(c, h, idx, tokens, out, out_w, ws, timeout_ns, waited);
    }
}

}  // namespace

void launch_combine_recv(const EpConfig& c, const p2p::HeapView& h, const int32_t* idx, int tokens, void* out,
                         const EpWorkspace& ws, uint64_t timeout_ns, cudaStream_t s, int grid, float* out_w,
                         bool waited) {
    if (grid <= 0) grid = 8 * default_grid();
    if (out_w && !c.comb_weights) throw kiwi::error("combine_recv: the op's combine slots carry no weights");
    uint8_t* o = static_cast<uint8_t*>(out);
    const int wt = waited ? 1 : 0;
    switch (static_cast<CombDtype>(c.comb_dtype)) {
        case CombDtype::kBf16: launch_combine_recv_dt<0>(c, h, idx, tokens, o, out_w, ws, timeout_ns, s, grid, wt); break;
        case CombDtype::kF32: launch_combine_recv_dt<1>(c, h, idx, tokens, o, out_w, ws, timeout_ns, s, grid, wt); break;
        case CombDtype::kFp8: launch_combine_recv_dt<2>(c, h, idx, tokens, o, out_w, ws, timeout_ns, s, grid, wt); break;
        case CombDtype::kFp4: launch_combine_recv_dt<3>(c, h, idx, tokens, o, out_w, ws, timeout_ns, s, grid, wt); break;
    }
    KIWI_CUDA_CHECK(cudaGetLastError());
}

void launch_recv_compact(const EpConfig& c, const p2p::HeapView& h, const EpWorkspace& ws, int32_t* slot_compact,
                         int32_t* recv_count, cudaStream_t s) {
    recv_compact_kernel<<<1, 1024, 0, s>>>(c, h, ws, slot_compact, recv_count);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

void launch_gather_rows(const EpConfig& c, const p2p::HeapView& h, const EpWorkspace& ws,
                        const int32_t* slot_compact, uint8_t* out_rows, uint8_t* out_scales, int32_t* out_idx,
                        float* out_w, int32_t* out_src_pos, cudaStream_t s) {
    gather_rows_kernel<<<2 * default_grid(), kThreads, 0, s>>>(c, h, ws, slot_compact, out_rows, out_scales, out_idx,
                                                              out_w, out_src_pos);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

void launch_combine_rows(const EpConfig& c, const p2p::HeapView& h, const void* rows, const float* weights,
                         const int32_t* src_pos, const int32_t* recv_count, const EpWorkspace& ws, cudaStream_t s) {
    if ((reinterpret_cast<uintptr_t>(rows) & 15u) != 0) throw kiwi::error("combine_rows: rows must be 16-byte aligned");
    if (weights && !c.comb_weights) throw kiwi::error("combine_rows: the op's combine slots carry no weights");
    combine_rows_kernel<<<2 * default_grid(), kThreads, 0, s>>>(c, h, static_cast<const uint8_t*>(rows), weights,
                                                               src_pos, recv_count, ws);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

}  // namespace kiwi::ep
