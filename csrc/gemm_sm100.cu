// Grouped BF16 GEMM on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
//   for each group g:  C[off_g : off_g + rows_g, :] = epilogue( A[off_g : .., :K] . B[g]^T )
//
// A is [total_rows, K] bf16 (K-major), B is [G * N, K] bf16 (K-major, one
// N x K matrix per group), C is bf16.  Group row counts live on the device
// (the MoE router fills them), so the tile schedule is built on the device
// and nothing here synchronises with the host: the launch is graph-capturable.
//
// Kernel shape (one CTA per SM, persistent over tiles):
//   warp 0       TMA producer: 128x64 A tile + BNx64 B tile per stage (SW128)
//   warp 1       TMEM owner + MMA issuer: tcgen05.mma kind::f16, M=128, N=BN, K=16
//   warps 2..5   epilogue: tcgen05.ld 32 columns at a time, optional SwiGLU /
//                per-row scale, bf16 stores
//   4 smem stages (A 16 KB + B 32 KB each), two TMEM accumulators of BN
//   columns so the epilogue of tile i overlaps the MMAs of tile i+1.
// Every mbarrier wait is bounded; a timeout sets *error and the CTA unwinds
// and frees its TMEM.
//
// SwiGLU epilogue: B rows of tile n hold [gate rows 128n..128n+127 |
// up rows 128n..128n+127] (interleave_gate_up() builds that layout), so one
// accumulator tile holds both halves and the epilogue writes silu(g) * u.
#include <cuda.h>

#include <atomic>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "kiwi/ep/quant.cuh"
#include "kiwi/ep/debug_timing.hpp"
#include "kiwi/gemm/grouped_gemm.hpp"
#include "kiwi/p2p/driver.hpp"
#include "kiwi/p2p/heap.hpp"
#include "kiwi/sm100.cuh"

namespace kiwi::gemm {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kStages = 4;
constexpr int kScatterStages = 4;
constexpr int kThreads = 192;
constexpr int kGatherThreads = 320;  // + 4 warps that gather and dequantise A
constexpr int kGatherDepth = 3;      // cp.async staging entries per gathering thread

/// Staged bytes per A row and k-block: FP8 64 data + 4 scale, NVFP4 32 data +
/// 4 block scales (padded to 16-byte multiples for cp.async).
template <int GQ>
constexpr int gather_row_bytes() { return GQ == 1 ? 80 : (GQ == 2 ? 48 : 0); }

enum Epi : int { kEpiStore = 0, kEpiSwiGLU = 1, kEpiScatter = 2 };

static_assert(kScatterMaxRanks == p2p::kMaxRanks, "ScatterArgs holds one base per rank");

/// Shared memory of one CTA: STAGES x (A tile + B tile), then (scatter
/// epilogue only) a bf16 staging tile per epilogue warp holding 32 rows of
/// BN/2 columns (256 bytes each, 16-byte chunks XOR-swizzled by row so that
/// both the row-per-thread writes and the row-wise reads are conflict-free),
/// then the barriers.
template <int BN, int STAGES = kStages, bool STAGING = false, int GQ = -1, int BKT = kBK>
struct Smem {
    static constexpr int kABytes = kBM * BKT * 2;
    static constexpr int kBBytes = BN * BKT * 2;
    // BKT = 128: each operand's stage holds two 64-column, 128-byte-swizzled
    // sub-tiles back to back (one TMA box each).
    static constexpr int kASub = kBM * 64 * 2;
    static constexpr int kBSub = BN * 64 * 2;
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kStgStride = BN;  // BN/2 bf16 columns = BN bytes per staged row
    static constexpr int kStgOffset = STAGES * kStageBytes;
    static constexpr int kStgBytes = STAGING ? 4 * 32 * kStgStride : 0;
    static constexpr int kGRow = gather_row_bytes<GQ>();
    static constexpr int kGStgOffset = kStgOffset + kStgBytes;
    static constexpr int kGStgBytes = GQ >= 0 ? kGatherDepth * kBM * kGRow : 0;
    static constexpr int kBarOffset = kGStgOffset + kGStgBytes;
    static constexpr int kBytes = kBarOffset + 256 + 1024;  // barriers + tmem slot + alignment slack
};

__device__ __forceinline__ void locate_tile(const int32_t* tile_prefix, int num_groups, int n_tiles, int tile,
                                            int& g, int& m_tile, int& n_tile) {
    int lo = 0, hi = num_groups - 1;
    while (lo < hi) {  // first g with tile_prefix[g + 1] > tile
        const int mid = (lo + hi) >> 1;
        if (__ldg(&tile_prefix[mid + 1]) > tile) hi = mid;
        else lo = mid + 1;
    }
    g = lo;
    // n-tile outermost within a group: the m-tiles that share one B (weight)
    // tile are adjacent in the schedule, run concurrently on neighbouring SMs
    // and read that tile from L2 instead of HBM.
    const int local = tile - __ldg(&tile_prefix[g]);
    const int m_tiles = (__ldg(&tile_prefix[g + 1]) - __ldg(&tile_prefix[g])) / n_tiles;
    n_tile = local / m_tiles;
    m_tile = local - n_tile * m_tiles;
}

/// One past the last row of group g (group_end, when given, bounds one pass of a split GEMM).
__device__ __forceinline__ int group_end_row(const GroupedArgs& p, int g) {
    return p.group_end ? __ldg(&p.group_end[g]) : __ldg(&p.group_offset[g + 1]);
}

/// Rows of group g that tile row block mt still covers (above kBM: a full tile).
__device__ __forceinline__ int tile_rows_left(const GroupedArgs& p, int g, int mt) {
    return group_end_row(p, g) - __ldg(&p.group_offset[g]) - mt * kBM;
}

/// Row of the tile whose accumulator is in `lane` of TMEM lane quadrant q, -1
/// for none: an M = 128 accumulator fills all 32 lanes of each quadrant, an
/// M = 64 one the first 16 (rows 16q..16q+15).
__device__ __forceinline__ int acc_row(int q, int lane, bool m64) {
    if (!m64) return q * 32 + lane;
    return lane < 16 ? q * 16 + lane : -1;
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

__device__ __forceinline__ void store_row32(__nv_bfloat16* dst, const float (&v)[32]) {
    uint4 out[4];
    uint32_t* w = reinterpret_cast<uint32_t*>(out);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < 4; ++i) d[i] = out[i];
}

/// Scatter epilogue of one 256-column accumulator tile for the 32 rows of the
/// calling warp (TMEM lane quadrant = the warp's rows): per half tile (128
/// columns) the warp stages its rows, routing-weight scaled, as bf16 in
/// XOR-swizzled shared memory, then stores them as 256-byte row segments (16
/// lanes per row, two rows per instruction) straight into each row's
/// destination (`my_dst` = (rank << 48) | byte offset, -1 = none) in the
/// ranks' heaps.  `release()` runs once the accumulator has been read, before
/// the second half's stores, so the next tile's MMAs overlap them.
template <typename Release>
__device__ __forceinline__ void scatter_tile(uint32_t taddr, uint8_t* stg, int64_t my_dst, float scale, int nt,
                                             uint8_t* const* s_base, Release&& release) {
    constexpr int BN = 256;
    constexpr int kStride = BN;  // BN / 2 bf16 columns = BN bytes per staged row
    const int lane = threadIdx.x & 31;
    const int half_lane = lane & 15;
#pragma unroll 1
    for (int half = 0; half < 2; ++half) {
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 32) {
            float v[32];
            sm100::tmem_ld_32cols(taddr + half * (BN / 2) + c, v);
            uint32_t w[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                __nv_bfloat162 hv = __floats2bfloat162_rn(v[2 * i] * scale, v[2 * i + 1] * scale);
                w[i] = *reinterpret_cast<uint32_t*>(&hv);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int chunk = (c / 8 + j) ^ (lane & 15);
                *reinterpret_cast<uint4*>(stg + lane * kStride + chunk * 16) =
                    make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
            }
        }
        if (half == 1) release();
        __syncwarp();
#pragma unroll 1
        for (int rr = 0; rr < 32; rr += 2) {
            const int row = rr + (lane >> 4);
            const long long d = __shfl_sync(0xffffffffu, static_cast<long long>(my_dst), row);
            if (d >= 0) {
                const int rank = static_cast<int>(d >> 48);
                uint8_t* dst = s_base[rank] + (d & kScatterOffMask) +
                               (static_cast<int64_t>(nt) * BN + half * (BN / 2)) * 2 + half_lane * 16;
                const uint4 val =
                    *reinterpret_cast<const uint4*>(stg + row * kStride + ((half_lane ^ (row & 15)) * 16));
                asm volatile("st.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "r"(val.x), "r"(val.y),
                             "r"(val.z), "r"(val.w)
                             : "memory");
            }
        }
        __syncwarp();
    }
}

/// Completion of a scatter GEMM: every CTA that did not abort releases its
/// stores at system scope and counts itself; the last one publishes
/// (epoch << 32) | 1 to every rank's flag.  With skip_signal (the first pass of
/// a split GEMM, ordered before the second on its stream) the CTA only fences.
/// Thread 0 only.
__device__ __forceinline__ void scatter_done(const ScatterArgs& sc, uint8_t* const* s_base) {
    asm volatile("fence.sc.sys;" ::: "memory");
    if (sc.skip_signal) return;  // a later pass of the same GEMM publishes the round
    const uint32_t prev = atomicAdd(sc.done_ctas, 1u);
    if (prev == gridDim.x - 1) {
        asm volatile("fence.sc.sys;" ::: "memory");
        const uint64_t v = (static_cast<uint64_t>(*reinterpret_cast<const volatile uint32_t*>(sc.epoch)) << 32) | 1u;
        for (int r = 0; r < sc.world; ++r) {
            asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(s_base[r] + sc.flag_off), "l"(v) : "memory");
        }
        *reinterpret_cast<volatile uint32_t*>(sc.done_ctas) = 0;
    }
}

template <int BN, int EPI, int STAGES, int GQ = -1, int BKT = kBK>
__global__ void __launch_bounds__(GQ >= 0 ? kGatherThreads : kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                        GroupedArgs p, const __grid_constant__ ScatterArgs sc, const __grid_constant__ GatherArgs ga) {
    constexpr int kStages = STAGES;
    constexpr int kBK = BKT;  // K per stage (64: 128-byte swizzle, 32: 64-byte swizzle, 128: two 64-column boxes)
    static_assert(GQ < 0 || BKT == 64, "the gathering producer writes 128-byte rows");
    using S = Smem<BN, STAGES, EPI == kEpiScatter, GQ, BKT>;
    __shared__ uint8_t* s_base[kScatterMaxRanks];
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kBarOffset);
    uint64_t* empty = full + kStages;
    uint64_t* tmem_full = empty + kStages;
    uint64_t* tmem_empty = tmem_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + 2);
    __shared__ int s_abort;

    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    const int n_tiles = p.n / BN;
    const int k_blocks = p.k / kBK;
    const int total_tiles = __ldg(&p.tile_prefix[p.num_groups]);

    if constexpr (EPI == kEpiScatter) {
        if (threadIdx.x < kScatterMaxRanks) s_base[threadIdx.x] = sc.base[threadIdx.x];
    }
    if (threadIdx.x == 0) {
        s_abort = 0;
        for (int s = 0; s < kStages; ++s) {
            // Gathered A: the TMA thread's arrival (B bytes) + one per A row.
            sm100::mbar_init(&full[s], GQ >= 0 ? 1 + kBM : 1);
            sm100::mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            sm100::mbar_init(&tmem_full[a], 1);
            sm100::mbar_init(&tmem_empty[a], 128);
        }
        sm100::fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        if constexpr (GQ < 0) sm100::tma_prefetch_desc(&tmap_a);
        sm100::tma_prefetch_desc(&tmap_b);
    }
    if (warp == 1) sm100::tmem_alloc(tmem_slot, 2 * BN);
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    if (threadIdx.x == 0) ep::span_start(p.span);

    auto fail = [&](uint32_t code) {
        *reinterpret_cast<volatile int*>(&s_abort) = 1;
        if (p.error) atomicCAS(p.error, 0u, code);
    };

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int64_t n_prod = 0;
            for (int tile = blockIdx.x; tile < total_tiles && !*reinterpret_cast<volatile int*>(&s_abort); tile += gridDim.x) {
                int g, mt, nt;
                locate_tile(p.tile_prefix, p.num_groups, n_tiles, tile, g, mt, nt);
                const int row0 = __ldg(&p.group_offset[g]) + mt * kBM;
                // B row of k-block 0 in either layout (row-major: x = kb * kBK
                // at brow0; blocked: x = 0 at brow0 + kb * BN).
                const int brow0 = p.b_blocked ? (g * n_tiles + nt) * k_blocks * BN : g * p.n + nt * BN;
                for (int kb = 0; kb < k_blocks; ++kb) {
                    const uint64_t tw0 = p.trace ? clock64() : 0;
                    if (!sm100::mbar_wait(&empty[stage], phase ^ 1)) {
                        fail(1);
                        break;
                    }
                    if (p.trace && blockIdx.x == 0 && n_prod < p.trace_capacity) {
                        p.trace[n_prod * kTraceSlots + 2] = tw0;
                        p.trace[n_prod * kTraceSlots + 3] = clock64();
                    }
                    ++n_prod;
                    uint8_t* sa = smem + stage * S::kStageBytes;
                    uint8_t* sb = sa + S::kABytes;
                    if constexpr (GQ >= 0) {
                        sm100::mbar_arrive_expect_tx(&full[stage], S::kBBytes);
                    } else {
                        sm100::mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
                        sm100::tma_load_2d(sa, &tmap_a, &full[stage], kb * kBK, row0);
                        if constexpr (BKT == 128) {
                            sm100::tma_load_2d(sa + S::kASub, &tmap_a, &full[stage], kb * kBK + 64, row0);
                        }
                    }
                    if constexpr (BKT == 64) {
                        if (p.b_blocked) sm100::tma_load_2d(sb, &tmap_b, &full[stage], 0, brow0 + kb * BN);
                        else sm100::tma_load_2d(sb, &tmap_b, &full[stage], kb * kBK, brow0);
                    } else {
                        sm100::tma_load_2d(sb, &tmap_b, &full[stage], kb * kBK, brow0);
                    }
                    if constexpr (BKT == 128) {
                        sm100::tma_load_2d(sb + S::kBSub, &tmap_b, &full[stage], kb * kBK + 64, brow0);
                    }
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc128 = sm100::idesc_bf16_f32(kBM, BN);
            const uint32_t idesc64 = sm100::idesc_bf16_f32(64, BN);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            int64_t n_mma = 0;
            for (int tile = blockIdx.x; tile < total_tiles && !*reinterpret_cast<volatile int*>(&s_abort); tile += gridDim.x) {
                uint32_t idesc = idesc128;
                if (p.m64_tails) {
                    int g, mt, nt;
                    locate_tile(p.tile_prefix, p.num_groups, n_tiles, tile, g, mt, nt);
                    if (tile_rows_left(p, g, mt) <= 64) idesc = idesc64;
                }
                if (!sm100::mbar_wait(&tmem_empty[acc], acc_phase ^ 1)) {
                    fail(2);
                    break;
                }
                sm100::tc_fence_after();
                const uint32_t d = tmem_base + acc * BN;
                bool ok = true;
                for (int kb = 0; kb < k_blocks; ++kb) {
                    const uint64_t tw0 = p.trace ? clock64() : 0;
                    if (!sm100::mbar_wait(&full[stage], phase)) {
                        fail(3);
                        ok = false;
                        break;
                    }
                    if (p.trace && blockIdx.x == 0 && n_mma < p.trace_capacity) {
                        p.trace[n_mma * kTraceSlots + 0] = tw0;
                        p.trace[n_mma * kTraceSlots + 1] = clock64();
                    }
                    ++n_mma;
                    sm100::tc_fence_after();
                    uint8_t* sa = smem + stage * S::kStageBytes;
                    uint8_t* sb = sa + S::kABytes;
                    const uint64_t adesc = sm100::kmajor_desc<BKT>(sa);
                    const uint64_t bdesc = sm100::kmajor_desc<BKT>(sb);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk) {
                        // +32 bytes of K per step inside the swizzle atom; with
                        // BKT = 128, steps 4..7 move to the second sub-tile (the
                        // descriptor's start address is in 16-byte units).
                        const int sub = BKT == 128 ? kk >> 2 : 0;
                        const int w = BKT == 128 ? kk & 3 : kk;
                        const uint64_t ad = adesc + static_cast<uint64_t>(sub * (S::kASub >> 4) + 2 * w);
                        const uint64_t bd = bdesc + static_cast<uint64_t>(sub * (S::kBSub >> 4) + 2 * w);
                        sm100::mma_bf16(d, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
                    }
                    sm100::mma_commit(&empty[stage]);
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                sm100::mma_commit(&tmem_full[acc]);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1;
                }
            }
        }
    } else if (warp >= 6) {
        if constexpr (GQ >= 0) {
            // Gathering A producer: thread r owns row r of every A tile.  Its
            // cp.async copies of (row, k-block) run kGatherDepth - 1 items
            // ahead of the dequantisation into the stage's swizzled A tile.
            const int r = (warp - 6) * 32 + lane;
            uint8_t* gstg = smem + S::kGStgOffset;
            auto row_slot_of = [&](int tile) -> int64_t {
                int g, mt, nt;
                locate_tile(p.tile_prefix, p.num_groups, n_tiles, tile, g, mt, nt);
                const int g_off = __ldg(&p.group_offset[g]);
                const int rr = mt * kBM + r;
                if (rr >= group_end_row(p, g) - g_off || g_off + rr >= p.max_rows) return -1;
                return __ldg(&ga.row_slot[g_off + rr]);
            };
            int i_tile = blockIdx.x, i_kb = 0;
            int64_t i_slot = i_tile < total_tiles ? row_slot_of(i_tile) : -1;
            uint32_t n_issued = 0;
            auto issue = [&]() {
                if (i_tile < total_tiles) {
                    uint8_t* dst = gstg + (n_issued % kGatherDepth) * (kBM * S::kGRow) + r * S::kGRow;
                    if (i_slot >= 0) {
                        const uint8_t* row = ga.base + ga.off_row + static_cast<uint64_t>(i_slot) * ga.row_bytes;
                        const uint8_t* scl = ga.base + ga.off_scale + static_cast<uint64_t>(i_slot) * ga.scale_bytes;
                        if constexpr (GQ == 1) {
#pragma unroll
                            for (int j = 0; j < 4; ++j) sm100::cp_async_16(dst + 16 * j, row + i_kb * 64 + 16 * j);
                            sm100::cp_async_4(dst + 64, scl + 4 * (i_kb / 2));
                        } else {
                            sm100::cp_async_16(dst, row + i_kb * 32);
                            sm100::cp_async_16(dst + 16, row + i_kb * 32 + 16);
                            sm100::cp_async_4(dst + 32, scl + 4 + 4 * i_kb);
                        }
                    }
                    if (++i_kb == k_blocks) {
                        i_kb = 0;
                        i_tile += gridDim.x;
                        i_slot = i_tile < total_tiles ? row_slot_of(i_tile) : -1;
                    }
                }
                sm100::cp_async_commit();  // one group per item, empty at the tail
                ++n_issued;
            };
#pragma unroll 1
            for (int d = 0; d < kGatherDepth - 1; ++d) issue();
            int stage = 0;
            uint32_t phase = 0;
            uint32_t n_done = 0;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < total_tiles && !*reinterpret_cast<volatile int*>(&s_abort);
                 tile += gridDim.x) {
                const int64_t slot = row_slot_of(tile);
                float row_scale = 1.0f;
                if constexpr (GQ == 2) {
                    if (slot >= 0) {
                        row_scale = __ldg(reinterpret_cast<const float*>(
                            ga.base + ga.off_scale + static_cast<uint64_t>(slot) * ga.scale_bytes));
                    }
                }
#pragma unroll 1
                for (int kb = 0; kb < k_blocks; ++kb) {
                    issue();
                    sm100::cp_async_wait<kGatherDepth - 1>();
                    if (!sm100::mbar_wait(&empty[stage], phase ^ 1)) {
                        fail(5);
                        ok = false;
                        break;
                    }
                    const uint8_t* src = gstg + (n_done % kGatherDepth) * (kBM * S::kGRow) + r * S::kGRow;
                    uint4 out[8];
                    if (slot < 0) {
#pragma unroll
                        for (int c = 0; c < 8; ++c) out[c] = make_uint4(0, 0, 0, 0);
                    } else if constexpr (GQ == 1) {
                        const float scl = *reinterpret_cast<const float*>(src + 64);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            uint4 o[2];
                            ep::dequant_fp8_16(*reinterpret_cast<const uint4*>(src + 16 * j), scl, o);
                            out[2 * j] = o[0];
                            out[2 * j + 1] = o[1];
                        }
                    } else {
                        const uint32_t sbs = *reinterpret_cast<const uint32_t*>(src + 32);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const __half_raw sh =
                                __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>((sbs >> (8 * j)) & 0xffu),
                                                        __NV_E4M3);
                            const float bs = __half2float(*reinterpret_cast<const __half*>(&sh)) * row_scale;
                            uint4 o[2];
                            ep::dequant_fp4_16(*reinterpret_cast<const uint2*>(src + 8 * j), bs, o);
                            out[2 * j] = o[0];
                            out[2 * j + 1] = o[1];
                        }
                    }
                    // 128-byte swizzle: 16-byte chunk c of row r goes to chunk c ^ (r % 8).
                    uint8_t* arow = smem + stage * S::kStageBytes + r * 128;
#pragma unroll
                    for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(arow + ((c ^ (r & 7)) * 16)) = out[c];
                    sm100::fence_proxy_async_smem();
                    sm100::mbar_arrive(&full[stage]);
                    ++n_done;
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            sm100::cp_async_wait<0>();
        }
    } else {
        // Epilogue: warps 2..5; TMEM lane quadrant = warp % 4.
        const int q = warp & 3;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int tile = blockIdx.x; tile < total_tiles && !*reinterpret_cast<volatile int*>(&s_abort); tile += gridDim.x) {
            int g, mt, nt;
            locate_tile(p.tile_prefix, p.num_groups, n_tiles, tile, g, mt, nt);
            if (!sm100::mbar_wait(&tmem_full[acc], acc_phase)) {
                fail(4);
                break;
            }
            sm100::tc_fence_after();
            const int g_off = __ldg(&p.group_offset[g]);
            const int g_rows = group_end_row(p, g) - g_off;
            const int row_in_tile = acc_row(q, lane, p.m64_tails && g_rows - mt * kBM <= 64);
            const int r = mt * kBM + row_in_tile;
            const int64_t out_row = static_cast<int64_t>(g_off) + r;
            const bool valid = row_in_tile >= 0 && r < g_rows && out_row < p.max_rows;
            const float scale = (valid && p.row_scale) ? p.row_scale[out_row] : 1.0f;
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
            if constexpr (EPI == kEpiSwiGLU) {
                __nv_bfloat16* crow = p.c + out_row * p.ldc + nt * (BN / 2);
#pragma unroll 1
                for (int c = 0; c < BN / 2; c += 32) {
                    float gv[32], uv[32];
                    sm100::tmem_ld_32cols(taddr + c, gv);
                    sm100::tmem_ld_32cols(taddr + BN / 2 + c, uv);
#pragma unroll
                    for (int i = 0; i < 32; ++i) gv[i] = silu(gv[i]) * uv[i] * scale;
                    if (valid) store_row32(crow + c, gv);
                }
                sm100::tc_fence_before();
                sm100::mbar_arrive(&tmem_empty[acc]);
            } else if constexpr (EPI == kEpiStore) {
                __nv_bfloat16* crow = p.c + out_row * p.ldc + nt * BN;
#pragma unroll 1
                for (int c = 0; c < BN; c += 32) {
                    float v[32];
                    sm100::tmem_ld_32cols(taddr + c, v);
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] *= scale;
                    if (valid) store_row32(crow + c, v);
                }
                sm100::tc_fence_before();
                sm100::mbar_arrive(&tmem_empty[acc]);
            } else {
                // Scatter: per half tile (BN/2 columns) stage the warp's 32
                // rows in shared memory, then store them as 256-byte row
                // segments (16 lanes per row, two rows per instruction) straight
                // into the destination ranks' heaps, so the NVLink traffic of
                // tile i overlaps the MMAs of tile i+1.  The accumulator is
                // released as soon as its second half has been read.
                static_assert(BN == 256, "scatter staging assumes 256-column tiles");
                uint8_t* stg = smem + S::kStgOffset + q * 32 * S::kStgStride;
                const int64_t my_dst = valid ? __ldg(&sc.row_dst[out_row]) : -1;
                scatter_tile(taddr, stg, my_dst, scale, nt, s_base, [&] {
                    sm100::tc_fence_before();
                    sm100::mbar_arrive(&tmem_empty[acc]);
                });
            }
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    if (warp == 1) sm100::tmem_dealloc(tmem_base, 2 * BN);
    if constexpr (EPI == kEpiScatter) {
        // Completion: every CTA releases its stores at system scope and counts
        // itself; the last one publishes (epoch << 32) | 1 to every rank.  A CTA
        // that aborted does not count, so the receivers' bounded waits report it.
        if (threadIdx.x == 0 && !*reinterpret_cast<volatile int*>(&s_abort)) scatter_done(sc, s_base);
    }
    if (threadIdx.x == 0) ep::span_end(p.span);
}


// ---------------------------------------------------------------------------
// 2-SM variant: a cluster of two CTAs computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2 (M = 256 across the pair).  Each CTA loads its 128
// rows of A and its 128-row half of the B tile, so a CTA moves 32 KB per
// k-block for 128 x 256 x 64 MACs instead of 48 KB: the L2 -> SMEM traffic per
// MMA drops by a third.  The leader (cluster rank 0) owns the full barriers
// (both CTAs' TMA loads complete on them) and issues the MMAs; commits arrive
// on both CTAs' barriers through their cluster addresses; each CTA drains its
// own TMEM (its 128 rows x 256 columns).  Used when experts get >= 256 rows.
// ---------------------------------------------------------------------------

constexpr int kPairStages = 6;
constexpr int kPairBM = 256;  // rows per pair tile (128 per CTA)
constexpr int kPairBN = 256;

/// Shared memory of one CTA of the pair: kPairStages x (A half + B half), then
/// (scatter epilogue) one 32-row x 128-column bf16 staging tile per epilogue
/// warp, then the barriers.  6 x 32 KB + 32 KB + 1.25 KB fits the 227 KB limit.
template <bool STAGING = false>
struct PairSmem {
    static constexpr int kABytes = 128 * kBK * 2;     // this CTA's 128 rows of A
    static constexpr int kBBytes = 128 * kBK * 2;     // this CTA's half of the B tile
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kStgOffset = kPairStages * kStageBytes;
    static constexpr int kStgStride = kPairBN;        // 128 bf16 columns = 256 bytes per staged row
    static constexpr int kStgBytes = STAGING ? 4 * 32 * kStgStride : 0;
    static constexpr int kBarOffset = kStgOffset + kStgBytes;
    static constexpr int kBytes = kBarOffset + 256 + 1024;
};
static_assert(PairSmem<true>::kBytes <= 227 * 1024, "pair scatter kernel exceeds the shared-memory limit");

template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    grouped_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                             GroupedArgs p, const __grid_constant__ ScatterArgs sc) {
    constexpr bool SWIGLU = EPI == kEpiSwiGLU;
    using S = PairSmem<EPI == kEpiScatter>;
    __shared__ uint8_t* s_base[kScatterMaxRanks];
    if constexpr (EPI == kEpiScatter) {
        if (threadIdx.x < kScatterMaxRanks) s_base[threadIdx.x] = sc.base[threadIdx.x];
    }
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kBarOffset);
    uint64_t* empty = full + kPairStages;
    uint64_t* tmem_full = empty + kPairStages;
    uint64_t* tmem_empty = tmem_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + 2);
    __shared__ int s_abort;

    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    const uint32_t crank = sm100::cluster_ctarank();
    const bool leader = crank == 0;
    const int cluster = blockIdx.x / 2;
    const int nclusters = gridDim.x / 2;
    const int n_tiles = p.n / kPairBN;
    const int k_blocks = p.k / kBK;
    const int total_tiles = __ldg(&p.tile_prefix[p.num_groups]);

    if (threadIdx.x == 0) {
        s_abort = 0;
        for (int st = 0; st < kPairStages; ++st) {
            sm100::mbar_init(&full[st], 1);
            sm100::mbar_init(&empty[st], 1);
        }
        for (int a = 0; a < 2; ++a) {
            sm100::mbar_init(&tmem_full[a], 1);
            sm100::mbar_init(&tmem_empty[a], 8);  // 4 epilogue warps x 2 CTAs
        }
        sm100::fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        sm100::tma_prefetch_desc(&tmap_a);
        sm100::tma_prefetch_desc(&tmap_b);
    }
    if (warp == 1) sm100::tmem_alloc_pair(tmem_slot, 2 * kPairBN);
    sm100::tc_fence_before();
    __syncthreads();
    sm100::cluster_sync();  // both CTAs' barriers exist before any cross-CTA arrival
    sm100::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    if (threadIdx.x == 0) ep::span_start(p.span);

    auto abort_flag = [&]() { return *reinterpret_cast<volatile int*>(&s_abort) != 0; };
    auto fail = [&](uint32_t code) {
        *reinterpret_cast<volatile int*>(&s_abort) = 1;
        if (p.error) atomicCAS(p.error, 0u, code);
    };

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            for (int tile = cluster; tile < total_tiles && !abort_flag(); tile += nclusters) {
                int g, mt, nt;
                locate_tile(p.tile_prefix, p.num_groups, n_tiles, tile, g, mt, nt);
                const int row0 = __ldg(&p.group_offset[g]) + mt * kPairBM + static_cast<int>(crank) * 128;
                // This CTA's 128-row half of the B tile (blocked: of each
                // 256-row k-block box).
                const int brow0 = p.b_blocked ? (g * n_tiles + nt) * k_blocks * kPairBN + static_cast<int>(crank) * 128
                                              : g * p.n + nt * kPairBN + static_cast<int>(crank) * 128;
                for (int kb = 0; kb < k_blocks; ++kb) {
                    if (!sm100::mbar_wait(&empty[stage], phase ^ 1)) {
                        fail(11);
                        break;
                    }
                    uint8_t* sa = smem + stage * S::kStageBytes;
                    uint8_t* sb = sa + S::kABytes;
                    if (leader) sm100::mbar_arrive_expect_tx(&full[stage], 2 * S::kStageBytes);
                    const uint32_t bar = sm100::mapa(&full[stage], 0);
                    sm100::tma_load_2d_pair(sa, &tmap_a, bar, kb * kBK, row0);
                    if (p.b_blocked) sm100::tma_load_2d_pair(sb, &tmap_b, bar, 0, brow0 + kb * kPairBN);
                    else sm100::tma_load_2d_pair(sb, &tmap_b, bar, kb * kBK, brow0);
                    if (++stage == kPairStages) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            const uint32_t idesc = sm100::idesc_bf16_f32(kPairBM, kPairBN);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            for (int tile = cluster; tile < total_tiles && !abort_flag(); tile += nclusters) {
                if (!sm100::mbar_wait(&tmem_empty[acc], acc_phase ^ 1)) {
                    fail(12);
                    break;
                }
                sm100::tc_fence_after();
                const uint32_t d = tmem_base + acc * kPairBN;
                bool ok = true;
                for (int kb = 0; kb < k_blocks; ++kb) {
                    if (!sm100::mbar_wait(&full[stage], phase)) {
                        fail(13);
                        ok = false;
                        break;
                    }
                    sm100::tc_fence_after();
                    uint8_t* sa = smem + stage * S::kStageBytes;
                    uint8_t* sb = sa + S::kABytes;
                    const uint64_t adesc = sm100::sw128_kmajor_desc(sa);
                    const uint64_t bdesc = sm100::sw128_kmajor_desc(sb);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk) {
                        sm100::mma_bf16_pair(d, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb | kk) != 0 ? 1u : 0u);
                    }
                    sm100::mma_commit_pair(sm100::mapa(&empty[stage], 0));
                    sm100::mma_commit_pair(sm100::mapa(&empty[stage], 1));
                    if (++stage == kPairStages) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                sm100::mma_commit_pair(sm100::mapa(&tmem_full[acc], 0));
                sm100::mma_commit_pair(sm100::mapa(&tmem_full[acc], 1));
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1;
                }
            }
        }
    } else {
        const int q = warp & 3;
        const int row_in_tile = static_cast<int>(crank) * 128 + q * 32 + lane;
        const uint32_t empty_leader = sm100::mapa(&tmem_empty[0], 0);
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int tile = cluster; tile < total_tiles && !abort_flag(); tile += nclusters) {
            int g, mt, nt;
            locate_tile(p.tile_prefix, p.num_groups, n_tiles, tile, g, mt, nt);
            if (!sm100::mbar_wait(&tmem_full[acc], acc_phase)) {
                fail(14);
                break;
            }
            sm100::tc_fence_after();
            const int g_off = __ldg(&p.group_offset[g]);
            const int g_rows = group_end_row(p, g) - g_off;
            const int r = mt * kPairBM + row_in_tile;
            const int64_t out_row = static_cast<int64_t>(g_off) + r;
            const bool valid = r < g_rows && out_row < p.max_rows;
            const float scale = (valid && p.row_scale) ? p.row_scale[out_row] : 1.0f;
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * kPairBN;
            if constexpr (EPI == kEpiScatter) {
                uint8_t* stg = smem + S::kStgOffset + q * 32 * S::kStgStride;
                const int64_t my_dst = valid ? __ldg(&sc.row_dst[out_row]) : -1;
                scatter_tile(taddr, stg, my_dst, scale, nt, s_base, [&] {
                    sm100::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        sm100::mbar_arrive_cluster(empty_leader + acc * static_cast<uint32_t>(sizeof(uint64_t)));
                    }
                });
            } else if constexpr (SWIGLU) {
                __nv_bfloat16* crow = p.c + out_row * p.ldc + nt * (kPairBN / 2);
#pragma unroll 1
                for (int c = 0; c < kPairBN / 2; c += 32) {
                    float gv[32], uv[32];
                    sm100::tmem_ld_32cols(taddr + c, gv);
                    sm100::tmem_ld_32cols(taddr + kPairBN / 2 + c, uv);
#pragma unroll
                    for (int i = 0; i < 32; ++i) gv[i] = silu(gv[i]) * uv[i] * scale;
                    if (valid) store_row32(crow + c, gv);
                }
            } else {
                __nv_bfloat16* crow = p.c + out_row * p.ldc + nt * kPairBN;
#pragma unroll 1
                for (int c = 0; c < kPairBN; c += 32) {
                    float v[32];
                    sm100::tmem_ld_32cols(taddr + c, v);
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] *= scale;
                    if (valid) store_row32(crow + c, v);
                }
            }
            if constexpr (EPI != kEpiScatter) {  // the scatter epilogue released the accumulator itself
                sm100::tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    sm100::mbar_arrive_cluster(empty_leader + acc * static_cast<uint32_t>(sizeof(uint64_t)));
                }
            }
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::cluster_sync();  // neither CTA leaves while its peer may still touch its barriers
    sm100::tc_fence_after();
    if (warp == 1) sm100::tmem_dealloc_pair(tmem_base, 2 * kPairBN);
    if constexpr (EPI == kEpiScatter) {
        if (threadIdx.x == 0 && !abort_flag()) scatter_done(sc, s_base);
    }
    if (threadIdx.x == 0) ep::span_end(p.span);
}

/// One block: exclusive scan of group row counts -> offsets, and of the tile
/// counts -> tile_prefix.  Works for up to 1024 groups.
__global__ void build_schedule_kernel(const int32_t* counts, int num_groups, int n_tiles, int bm, int32_t* offsets,
                                      int32_t* tile_prefix) {
    __shared__ int32_t s_rows[1024];
    __shared__ int32_t s_tiles[1024];
    const int t = threadIdx.x;
    const int rows = t < num_groups ? counts[t] : 0;
    s_rows[t] = rows;
    s_tiles[t] = ((rows + bm - 1) / bm) * n_tiles;
    __syncthreads();
    for (int d = 1; d < blockDim.x; d <<= 1) {
        const int a = t >= d ? s_rows[t - d] : 0;
        const int b = t >= d ? s_tiles[t - d] : 0;
        __syncthreads();
        s_rows[t] += a;
        s_tiles[t] += b;
        __syncthreads();
    }
    if (t < num_groups) {
        offsets[t + 1] = s_rows[t];
        tile_prefix[t + 1] = s_tiles[t];
    }
    if (t == 0) {
        offsets[0] = 0;
        tile_prefix[0] = 0;
    }
}

/// One block of a power-of-two thread count >= num_groups: per group, full
/// 256-row tiles for the 2-SM pass and 128-row tail tiles for the 1-SM pass,
/// prefix-summed for one or two GEMMs.
__global__ void build_split_schedule_kernel(const int32_t* counts, int num_groups, int n_tiles1, int n_tiles2,
                                            SplitSchedule out) {
    __shared__ int32_t s_rows[1024];
    __shared__ int32_t s_pair[1024];
    __shared__ int32_t s_tail[1024];
    const int t = threadIdx.x;
    const int rows = t < num_groups ? counts[t] : 0;
    const int full = rows / 256;
    s_rows[t] = rows;
    s_pair[t] = full;
    s_tail[t] = (rows - 256 * full + 127) / 128;
    __syncthreads();
    for (int d = 1; d < blockDim.x; d <<= 1) {
        const int a = t >= d ? s_rows[t - d] : 0;
        const int b = t >= d ? s_pair[t - d] : 0;
        const int c = t >= d ? s_tail[t - d] : 0;
        __syncthreads();
        s_rows[t] += a;
        s_pair[t] += b;
        s_tail[t] += c;
        __syncthreads();
    }
    if (t < num_groups) {
        out.offsets[t + 1] = s_rows[t];
        out.pair_end[t] = s_rows[t] - rows + 256 * full;
        out.pair_tiles1[t + 1] = s_pair[t] * n_tiles1;
        out.tail_tiles1[t + 1] = s_tail[t] * n_tiles1;
        if (out.pair_tiles2) {
            out.pair_tiles2[t + 1] = s_pair[t] * n_tiles2;
            out.tail_tiles2[t + 1] = s_tail[t] * n_tiles2;
        }
    }
    if (t == 0) {
        out.offsets[0] = 0;
        out.pair_tiles1[0] = 0;
        out.tail_tiles1[0] = 0;
        if (out.pair_tiles2) {
            out.pair_tiles2[0] = 0;
            out.tail_tiles2[0] = 0;
        }
    }
}

}  // namespace

CUtensorMap make_tmap_bf16_2d(const void* ptr, uint64_t rows, uint64_t cols, uint32_t box_rows, uint32_t box_k) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (!encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q{};
        KIWI_CUDA_CHECK(cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !fn) throw kiwi::error("cuTensorMapEncodeTiled unavailable");
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0 || (cols * 2) % 16 != 0) {
        throw kiwi::error("make_tmap_bf16_2d: base and row stride must be 16-byte aligned");
    }
    CUtensorMap m;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 2};
    if (box_k != 64 && box_k != 32) throw kiwi::error("make_tmap_bf16_2d: box_k must be 64 or 32");
    const cuuint32_t box[2] = {box_k, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE,
                              box_k == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    p2p::check_cu(r, "cuTensorMapEncodeTiled");
    return m;
}

void build_schedule(const int32_t* counts, int num_groups, int n, int bn, int32_t* offsets, int32_t* tile_prefix,
                    cudaStream_t stream, int bm) {
    if (num_groups < 1 || num_groups > 1024) throw kiwi::error("build_schedule: 1..1024 groups");
    if (bm != kBM && bm != kPairBM) throw kiwi::error("build_schedule: bm must be 128 or 256");
    int threads = 32;
    while (threads < num_groups) threads <<= 1;
    build_schedule_kernel<<<1, threads, 0, stream>>>(counts, num_groups, n / bn, bm, offsets, tile_prefix);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

void build_split_schedule(const int32_t* counts, int num_groups, int n1, int n2, const SplitSchedule& out,
                          cudaStream_t stream) {
    if (num_groups < 1 || num_groups > 1024) throw kiwi::error("build_split_schedule: 1..1024 groups");
    if (n1 <= 0 || n1 % 256 || (out.pair_tiles2 && (n2 <= 0 || n2 % 256))) {
        throw kiwi::error("build_split_schedule: N must be a positive multiple of 256");
    }
    if (!out.offsets || !out.pair_end || !out.pair_tiles1 || !out.tail_tiles1 ||
        (out.pair_tiles2 == nullptr) != (out.tail_tiles2 == nullptr)) {
        throw kiwi::error("build_split_schedule: missing output arrays");
    }
    int threads = 32;
    while (threads < num_groups) threads <<= 1;
    build_split_schedule_kernel<<<1, threads, 0, stream>>>(counts, num_groups, n1 / 256, n2 > 0 ? n2 / 256 : 0, out);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

namespace {

constexpr int kMaxCachedDevices = 64;

int current_device() {
    int dev = 0;
    KIWI_CUDA_CHECK(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxCachedDevices) throw kiwi::error("grouped_gemm: device index beyond 64");
    return dev;
}

/// Raises `kernel`'s dynamic shared-memory limit to `smem` on the current
/// device.  The attribute is per device, so `done` keeps one bit per device;
/// two threads racing on the first launch both set it, which is harmless.
template <typename Kernel>
void raise_smem_limit(Kernel kernel, int smem, std::atomic<uint64_t>& done) {
    const uint64_t bit = 1ull << current_device();
    if (done.load(std::memory_order_acquire) & bit) return;
    KIWI_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    done.fetch_or(bit, std::memory_order_acq_rel);
}

}  // namespace

int num_sms() {
    static std::atomic<int> cached[kMaxCachedDevices] = {};
    const int dev = current_device();
    int n = cached[dev].load(std::memory_order_relaxed);
    if (n == 0) {
        KIWI_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
        cached[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

namespace {

template <int EPI, int STAGES, int GQ = -1, int BKT = kBK>
void launch_grouped(const CUtensorMap& tmap_a, const CUtensorMap& tmap_b, const GroupedArgs& args,
                    const ScatterArgs& sc, int grid, cudaStream_t stream, const GatherArgs& ga = GatherArgs{}) {
    constexpr int BN = 256;
    const int smem = Smem<BN, STAGES, EPI == kEpiScatter, GQ, BKT>::kBytes;
    static std::atomic<uint64_t> attr{0};
    raise_smem_limit(grouped_gemm_kernel<BN, EPI, STAGES, GQ, BKT>, smem, attr);
    grouped_gemm_kernel<BN, EPI, STAGES, GQ, BKT>
        <<<grid, GQ >= 0 ? kGatherThreads : kThreads, smem, stream>>>(tmap_a, tmap_b, args, sc, ga);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

void check_shape(const GroupedArgs& args) {
    if (args.n % 256 != 0 || args.k % kBK != 0) {
        throw kiwi::error("grouped_gemm: N must be a multiple of 256 and K of 64");
    }
}

}  // namespace

void grouped_gemm(const CUtensorMap& tmap_a, const CUtensorMap& tmap_b, const GroupedArgs& args, bool swiglu,
                  int grid, cudaStream_t stream) {
    check_shape(args);
    if (grid <= 0) grid = num_sms();
    const ScatterArgs none{};
    if (swiglu) launch_grouped<kEpiSwiGLU, kStages>(tmap_a, tmap_b, args, none, grid, stream);
    else launch_grouped<kEpiStore, kStages>(tmap_a, tmap_b, args, none, grid, stream);
}

constexpr int kBk32Stages = 9;   // 9 x 24 KB stages
constexpr int kBk128Stages = 2;  // 2 x 96 KB stages (half the stage hand-offs of BK 64 per FLOP)

void grouped_gemm_bk128(const CUtensorMap& tmap_a, const CUtensorMap& tmap_b, const GroupedArgs& args, bool swiglu,
                        int grid, cudaStream_t stream) {
    if (args.n % 256 != 0 || args.k % 128 != 0) {
        throw kiwi::error("grouped_gemm_bk128: N must be a multiple of 256 and K of 128");
    }
    if (args.b_blocked) throw kiwi::error("grouped_gemm_bk128: the blocked B layout needs 64-column k-blocks");
    if (grid <= 0) grid = num_sms();
    const ScatterArgs none{};
    if (swiglu) launch_grouped<kEpiSwiGLU, kBk128Stages, -1, 128>(tmap_a, tmap_b, args, none, grid, stream);
    else launch_grouped<kEpiStore, kBk128Stages, -1, 128>(tmap_a, tmap_b, args, none, grid, stream);
}

void grouped_gemm_bk32(const CUtensorMap& tmap_a32, const CUtensorMap& tmap_b32, const GroupedArgs& args,
                       bool swiglu, int grid, cudaStream_t stream) {
    if (args.n % 256 != 0 || args.k % 32 != 0) {
        throw kiwi::error("grouped_gemm_bk32: N must be a multiple of 256 and K of 32");
    }
    if (args.b_blocked) throw kiwi::error("grouped_gemm_bk32: the blocked B layout needs 64-column k-blocks");
    if (grid <= 0) grid = num_sms();
    const ScatterArgs none{};
    if (swiglu) launch_grouped<kEpiSwiGLU, kBk32Stages, -1, 32>(tmap_a32, tmap_b32, args, none, grid, stream);
    else launch_grouped<kEpiStore, kBk32Stages, -1, 32>(tmap_a32, tmap_b32, args, none, grid, stream);
}

void grouped_gemm_gather(const CUtensorMap& tmap_b, const GroupedArgs& args, const GatherArgs& ga, int grid,
                         cudaStream_t stream) {
    check_shape(args);
    if (!ga.base || !ga.row_slot) throw kiwi::error("grouped_gemm_gather: missing receive buffer or row slots");
    if (ga.row_bytes % 16 || ga.off_row % 16 || ga.scale_bytes % 16 || ga.off_scale % 16) {
        throw kiwi::error("grouped_gemm_gather: rows and scales must be 16-byte aligned");
    }
    if (grid <= 0) grid = num_sms();
    const ScatterArgs none{};
    // tmap_b stands in for the unused A map (the A tile is gathered).
    if (ga.quant == 1) {
        if (ga.row_bytes < args.k) throw kiwi::error("grouped_gemm_gather: FP8 rows shorter than K");
        launch_grouped<kEpiSwiGLU, kStages, 1>(tmap_b, tmap_b, args, none, grid, stream, ga);
    } else if (ga.quant == 2) {
        if (ga.row_bytes * 2 < args.k) throw kiwi::error("grouped_gemm_gather: NVFP4 rows shorter than K");
        launch_grouped<kEpiSwiGLU, kStages, 2>(tmap_b, tmap_b, args, none, grid, stream, ga);
    } else {
        throw kiwi::error("grouped_gemm_gather: quant must be 1 (FP8) or 2 (NVFP4)");
    }
}

void grouped_gemm_scatter(const CUtensorMap& tmap_a, const CUtensorMap& tmap_b, const GroupedArgs& args,
                          const ScatterArgs& sc, int grid, cudaStream_t stream) {
    check_shape(args);
    if (args.n * 2 % 512 != 0) throw kiwi::error("grouped_gemm_scatter: N must be a multiple of 256");
    if (!sc.row_dst || !sc.done_ctas || !sc.epoch) throw kiwi::error("grouped_gemm_scatter: missing arguments");
    if (sc.world < 1 || sc.world > kScatterMaxRanks) throw kiwi::error("grouped_gemm_scatter: world out of range");
    if (grid <= 0) grid = num_sms();
    launch_grouped<kEpiScatter, kScatterStages>(tmap_a, tmap_b, args, sc, grid, stream);
}

namespace {

template <int EPI>
void launch_pair(const CUtensorMap& tmap_a, const CUtensorMap& tmap_b_half, const GroupedArgs& args,
                 const ScatterArgs& sc, int grid, cudaStream_t stream) {
    if (args.n % kPairBN != 0 || args.k % kBK != 0) {
        throw kiwi::error("grouped_gemm_pair: N must be a multiple of 256 and K of 64");
    }
    const int smem = PairSmem<EPI == kEpiScatter>::kBytes;
    if (grid <= 0) grid = num_sms();
    grid &= ~1;  // whole clusters of two
    if (grid < 2) throw kiwi::error("grouped_gemm_pair: needs at least two SMs");
    static std::atomic<uint64_t> attr{0};
    raise_smem_limit(grouped_gemm_pair_kernel<EPI>, smem, attr);
    grouped_gemm_pair_kernel<EPI><<<grid, kThreads, smem, stream>>>(tmap_a, tmap_b_half, args, sc);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

}  // namespace

void grouped_gemm_pair(const CUtensorMap& tmap_a, const CUtensorMap& tmap_b_half, const GroupedArgs& args,
                       bool swiglu, int grid, cudaStream_t stream) {
    const ScatterArgs none{};
    if (swiglu) launch_pair<kEpiSwiGLU>(tmap_a, tmap_b_half, args, none, grid, stream);
    else launch_pair<kEpiStore>(tmap_a, tmap_b_half, args, none, grid, stream);
}

void grouped_gemm_pair_scatter(const CUtensorMap& tmap_a, const CUtensorMap& tmap_b_half, const GroupedArgs& args,
                               const ScatterArgs& sc, int grid, cudaStream_t stream) {
    if (!sc.row_dst || !sc.done_ctas || !sc.epoch) throw kiwi::error("grouped_gemm_pair_scatter: missing arguments");
    if (sc.world < 1 || sc.world > kScatterMaxRanks) throw kiwi::error("grouped_gemm_pair_scatter: world out of range");
    launch_pair<kEpiScatter>(tmap_a, tmap_b_half, args, sc, grid, stream);
}

KernelInfo gemm_pair_kernel_info(bool swiglu) {
    cudaFuncAttributes a{};
    if (swiglu) KIWI_CUDA_CHECK(cudaFuncGetAttributes(&a, grouped_gemm_pair_kernel<kEpiSwiGLU>));
    else KIWI_CUDA_CHECK(cudaFuncGetAttributes(&a, grouped_gemm_pair_kernel<kEpiStore>));
    return {static_cast<int>(a.localSizeBytes), a.numRegs, PairSmem<false>::kBytes};
}

KernelInfo gemm_pair_scatter_kernel_info() {
    cudaFuncAttributes a{};
    KIWI_CUDA_CHECK(cudaFuncGetAttributes(&a, grouped_gemm_pair_kernel<kEpiScatter>));
    return {static_cast<int>(a.localSizeBytes), a.numRegs, PairSmem<true>::kBytes};
}

KernelInfo gemm_kernel_info(bool swiglu) {
    cudaFuncAttributes a{};
    if (swiglu) KIWI_CUDA_CHECK(cudaFuncGetAttributes(&a, grouped_gemm_kernel<256, kEpiSwiGLU, kStages>));
    else KIWI_CUDA_CHECK(cudaFuncGetAttributes(&a, grouped_gemm_kernel<256, kEpiStore, kStages>));
    return {static_cast<int>(a.localSizeBytes), a.numRegs, Smem<256>::kBytes};
}

KernelInfo gemm_gather_kernel_info(int quant) {
    cudaFuncAttributes a{};
    if (quant == 2) {
        KIWI_CUDA_CHECK(cudaFuncGetAttributes(&a, grouped_gemm_kernel<256, kEpiSwiGLU, kStages, 2>));
        return {static_cast<int>(a.localSizeBytes), a.numRegs, Smem<256, kStages, false, 2>::kBytes};
    }
    KIWI_CUDA_CHECK(cudaFuncGetAttributes(&a, grouped_gemm_kernel<256, kEpiSwiGLU, kStages, 1>));
    return {static_cast<int>(a.localSizeBytes), a.numRegs, Smem<256, kStages, false, 1>::kBytes};
}

KernelInfo gemm_scatter_kernel_info() {
    cudaFuncAttributes a{};
    KIWI_CUDA_CHECK(cudaFuncGetAttributes(&a, grouped_gemm_kernel<256, kEpiScatter, kScatterStages>));
    return {static_cast<int>(a.localSizeBytes), a.numRegs, Smem<256, kScatterStages, true>::kBytes};
}

}  // namespace kiwi::gemm
