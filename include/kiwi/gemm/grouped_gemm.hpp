// Host API of the sm_100a grouped BF16 GEMM (csrc/gemm_sm100.cu).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "kiwi/common.hpp"

namespace kiwi::gemm {

struct GroupedArgs {
    const int32_t* group_offset;  // [G + 1] device: first row of each group in A and C
    const int32_t* tile_prefix;   // [G + 1] device: cumulative 128 x BN tiles per group
    int32_t num_groups;
    int32_t n;                    // B rows per group (C columns before SwiGLU halves them)
    int32_t k;
    // 1-SM kernel only, non-zero: a tile whose group has at most 64 rows left
    // runs M = 64 MMAs (half the tensor work of a mostly-padding tile, same
    // K order, so the result is bit-identical); its accumulator holds rows
    // 16q..16q+15 in TMEM lanes 32q..32q+15 of lane quadrant q.
    int32_t m64_tails;
    // Non-zero: B is in the blocked layout (kiwi_b200.ops.block_weights): the
    // 256-row x 64-column box of (group g, n-tile nt, k-block kb) is 32 KB of
    // contiguous memory at row ((g * N / 256 + nt) * K / 64 + kb) * 256 of a
    // [G * N * K / 64, 64] matrix, so a weight load reads whole DRAM pages
    // instead of 128-byte pieces one B row stride apart.  64-column k-blocks
    // only (not the bk = 32 / 128 variants).
    int32_t b_blocked;
    int32_t pad_;
    __nv_bfloat16* c;
    int64_t ldc;                  // C row stride, elements
    const float* row_scale;       // optional per-row factor applied in the epilogue
    uint32_t* error;              // device word: non-zero if a bounded wait ran out
    int64_t max_rows;             // rows C holds: rows at or past it are never stored
    // Optional pipeline trace of CTA 0 (null: off).  trace[0..n) of
    // kTraceSlots each: {mma_wait_full_start, mma_wait_full_end,
    // producer_wait_empty_start, producer_wait_empty_end} in SM clock cycles,
    // one slot per k-block in issue order; trace_capacity slots at most.
    uint64_t* trace;
    int64_t trace_capacity;
    // Optional kernel span (null: off): span[0] = ~(first CTA start) and
    // span[1] = last CTA end, %globaltimer ns, both updated with atomicMax
    // (the layout of one phase of kiwi::ep's debug timing buffer).
    uint64_t* span;
    // Optional [G] device: group g's rows end at group_end[g] instead of
    // group_offset[g + 1] (one pass of a GEMM split into full 256-row tiles and
    // tails; group_offset then only needs G entries).
    const int32_t* group_end;
};

inline constexpr int kTraceSlots = 4;

/// Scatter epilogue of the fused MoE combine (grouped_gemm_scatter): result
/// row r, scaled by row_scale[r] and converted to bf16, is stored at byte
/// offset (row_dst[r] & kScatterOffMask) of rank (row_dst[r] >> 48)'s heap
/// (base[rank], a peer mapping for other ranks); row_dst[r] < 0 drops the row.
/// When every CTA has finished, the last one stores (epoch << 32) | 1 with
/// release semantics at flag_off of every rank's heap.  done_ctas must be zero
/// at launch (the last CTA leaves it zero again).
inline constexpr int kScatterMaxRanks = 16;
inline constexpr uint64_t kScatterOffMask = (uint64_t{1} << 48) - 1;

struct ScatterArgs {
    uint8_t* base[kScatterMaxRanks];
    const int64_t* row_dst;
    uint32_t* done_ctas;
    const uint32_t* epoch;
    uint64_t flag_off;
    int32_t world;
    int32_t skip_signal;  // 1: fence this launch's stores and publish nothing (a split GEMM's first pass)
};

/// Gathering A producer (fused EP receive -> GEMM1): expert-major row i of A is
/// the dispatched row of slot row_slot[i], read in place from the receive
/// buffer and dequantised to bf16 in shared memory.  quant 1: FP8 e4m3 rows
/// of row_bytes at base + off_row + slot * row_bytes with fp32 scales per 128
/// columns at base + off_scale + slot * scale_bytes; quant 2: NVFP4 (e2m1
/// pairs per byte, an fp32 row scale then one e4m3 scale per 16 columns).
struct GatherArgs {
    const uint8_t* base;
    const int32_t* row_slot;
    uint64_t off_row;
    uint64_t off_scale;
    int32_t row_bytes;
    int32_t scale_bytes;
    int32_t quant;
    int32_t pad_;
};

struct KernelInfo {
    int local_bytes;
    int registers;
    int smem_bytes;
};

/// Tensor map of a row-major [rows, cols] bf16 matrix, box [box_rows, box_k]:
/// box_k 64 with the 128-byte swizzle (grouped_gemm and friends) or 32 with
/// the 64-byte swizzle (grouped_gemm_bk32), the layouts the kernels'
/// shared-memory descriptors expect.
CUtensorMap make_tmap_bf16_2d(const void* ptr, uint64_t rows, uint64_t cols, uint32_t box_rows,
                              uint32_t box_k = 64);

/// Builds group offsets and the tile prefix from per-group row counts (device).
/// `bm` = rows per tile: 128 for grouped_gemm, 256 for grouped_gemm_pair.
void build_schedule(const int32_t* counts, int num_groups, int n, int bn, int32_t* offsets, int32_t* tile_prefix,
                    cudaStream_t stream, int bm = 128);

/// Device arrays of a grouped GEMM split into a 2-SM pass over every group's
/// full 256-row tiles and a 1-SM pass over the remaining rows (< 256 per
/// group), for up to two GEMMs over the same row counts (different N).
struct SplitSchedule {
    int32_t* offsets;      // [G + 1] first row of each group
    int32_t* pair_end;     // [G] end of each group's full 256-row tiles (= start of its tail)
    int32_t* pair_tiles1;  // [G + 1] cumulative 256-row x 256-column tiles of GEMM 1
    int32_t* tail_tiles1;  // [G + 1] cumulative 128-row x 256-column tail tiles of GEMM 1
    int32_t* pair_tiles2;  // same for GEMM 2 (null: one GEMM)
    int32_t* tail_tiles2;
};

/// Fills a SplitSchedule from per-group row counts on the device (one block,
/// at most 1024 groups); n1 / n2: each GEMM's N (multiples of 256).
void build_split_schedule(const int32_t* counts, int num_groups, int n1, int n2, const SplitSchedule& out,
                          cudaStream_t stream);

/// Launches the persistent grouped GEMM (BN = 256).  `grid` <= 0: one CTA per SM.
void grouped_gemm(const CUtensorMap& tmap_a, const CUtensorMap& tmap_b, const GroupedArgs& args, bool swiglu,
                  int grid, cudaStream_t stream);

/// Variant with 32-column K stages (64-byte swizzle, 9 stages of 24 KB): more
/// lookahead per byte of shared memory for operand loads whose latency the
/// 4 x 48 KB stages of grouped_gemm do not cover.  Tensor maps from
/// make_tmap_bf16_2d(..., box_k = 32).  Same results as grouped_gemm (the
/// same K = 16 MMA sequence).
/// The 1-SM kernel with 128 columns of K per stage: two 64-column boxes per
/// operand (the default 128-byte-swizzled maps), 2 stages of 96 KB, the same
/// MMA order as grouped_gemm.  K must be a multiple of 128.
void grouped_gemm_bk128(const CUtensorMap& tmap_a, const CUtensorMap& tmap_b, const GroupedArgs& args, bool swiglu,
                        int grid, cudaStream_t stream);

void grouped_gemm_bk32(const CUtensorMap& tmap_a32, const CUtensorMap& tmap_b32, const GroupedArgs& args,
                       bool swiglu, int grid, cudaStream_t stream);

/// 2-SM variant (clusters of two CTAs, 256 x 256 tiles).  `tmap_b_half` must
/// have a box of 128 rows (each CTA loads half of the 256-row B tile); the
/// schedule must be built with bm = 256.
void grouped_gemm_pair(const CUtensorMap& tmap_a, const CUtensorMap& tmap_b_half, const GroupedArgs& args,
                       bool swiglu, int grid, cudaStream_t stream);

/// Grouped GEMM whose epilogue scatters rows to (remote) heaps and signals
/// completion (see ScatterArgs).  N must be a multiple of 256 (whole 512-byte
/// rows per tile); 4 pipeline stages plus 32 KB of half-row staging tiles.
void grouped_gemm_scatter(const CUtensorMap& tmap_a, const CUtensorMap& tmap_b, const GroupedArgs& args,
                          const ScatterArgs& sc, int grid, cudaStream_t stream);

/// GEMM1 with the SwiGLU epilogue whose A operand is gathered from the receive
/// buffer (GatherArgs) instead of a dense bf16 matrix; tmap_b as grouped_gemm.
void grouped_gemm_gather(const CUtensorMap& tmap_b, const GroupedArgs& args, const GatherArgs& ga, int grid,
                         cudaStream_t stream);

KernelInfo gemm_kernel_info(bool swiglu);
KernelInfo gemm_gather_kernel_info(int quant);
KernelInfo gemm_scatter_kernel_info();
KernelInfo gemm_pair_kernel_info(bool swiglu);
KernelInfo gemm_pair_scatter_kernel_info();

/// The 2-SM kernel (256-row tiles, cta_group::2) with the NVLink scatter
/// epilogue of grouped_gemm_scatter (same ScatterArgs, same completion
/// signal); tmap_b_half as grouped_gemm_pair.  Schedules with bm = 256.
void grouped_gemm_pair_scatter(const CUtensorMap& tmap_a, const CUtensorMap& tmap_b_half, const GroupedArgs& args,
                               const ScatterArgs& sc, int grid, cudaStream_t stream);
int num_sms();

}  // namespace kiwi::gemm
