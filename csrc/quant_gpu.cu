// Stand-alone block quantisation of bf16 rows with the EP dispatch kernel's
// arithmetic (kiwi/ep/quant.cuh), for callers that quantise outside the fused
// dispatch, such as the all-to-all EP transport: both transports then carry
// the same bytes.
//   FP8 1x128: one warp per 512-element chunk of a row; each lane converts 16
//              elements and eight lanes share one block scale.
//   NVFP4:     one warp per row; the row's fp32 scale amax / (448 * 6) comes
//              from a warp reduction, then each lane converts one 16-element
//              block (e4m3 block scale relative to the row scale, e2m1 codes).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "kiwi/common.hpp"
#include "kiwi/ep/quant.cuh"
#include "kiwi/ops/quant.hpp"

namespace kiwi::ops {

namespace {

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads) quant_fp8_rows_kernel(const __nv_bfloat16* __restrict__ x,
                                                                   uint8_t* __restrict__ codes,
                                                                   float* __restrict__ scales, int64_t rows,
                                                                   int hidden) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * kThreads) >> 5;
    const int chunks = (hidden + 511) / 512;
    const int64_t work = rows * chunks;
    for (int64_t w = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5; w < work; w += nwarps) {
        const int64_t r = w / chunks;
        const int e0 = static_cast<int>(w % chunks) * 512 + lane * 16;  // this lane's first element
        const bool valid = e0 < hidden;  // hidden % 128 == 0: a block's 8 lanes agree
        uint4 in[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
        if (valid) {
            const uint4* p = reinterpret_cast<const uint4*>(x + r * hidden + e0);
            in[0] = p[0];
            in[1] = p[1];
        }
        float scale;
        uint4 q;
        ep::quant_fp8_16(in, scale, q);  // warp-collective (block amax by shuffles)
        if (valid) {
            *reinterpret_cast<uint4*>(codes + r * hidden + e0) = q;
            if ((lane & 7) == 0) scales[r * (hidden / 128) + e0 / 128] = scale;
        }
    }
}

/// One warp per row.  The row scale is the dispatch kernel's (row amax over
/// the warp, IEEE-divided by 448 * 6); block scales and codes come from
/// ep::quant_fp4_16, so the bytes equal what the NVLink dispatch stores.
__global__ void __launch_bounds__(kThreads) quant_nvfp4_rows_kernel(const __nv_bfloat16* __restrict__ x,
                                                                     uint8_t* __restrict__ codes,
                                                                     uint8_t* __restrict__ scales, int64_t rows,
                                                                     int hidden, int scale_bytes) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * kThreads) >> 5;
    for (int64_t r = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5; r < rows; r += nwarps) {
        const __nv_bfloat16* xr = x + r * hidden;
        float amax = 0.f;
        for (int col = lane * 8; col < hidden; col += 256) {
            float f[8];
            ep::bf16x8_to_f32(*reinterpret_cast<const uint4*>(xr + col), f);
#pragma unroll
            for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(f[i]));
        }
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, d));
        const float row_scale = amax > 0.f ? amax / (ep::kFp8Max * ep::kFp4Max) : 0.f;
        uint8_t* sr = scales + r * scale_bytes;
        if (lane == 0) *reinterpret_cast<float*>(sr) = row_scale;
        for (int col = lane * 16; col < hidden; col += 512) {
            uint4 in[2];
            in[0] = *reinterpret_cast<const uint4*>(xr + col);
            in[1] = *reinterpret_cast<const uint4*>(xr + col + 8);
            uint8_t sb;
            uint2 q;
            ep::quant_fp4_16(in, row_scale, sb, q);
            sr[4 + col / 16] = sb;
            *reinterpret_cast<uint2*>(codes + r * (hidden / 2) + col / 2) = q;
        }
        for (int o = 4 + hidden / 16 + lane; o < scale_bytes; o += 32) sr[o] = 0;  // padding
    }
}

int grid_for(int64_t warps) {
    int dev = 0, sms = 0;
    KIWI_CUDA_CHECK(cudaGetDevice(&dev));
    KIWI_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    return static_cast<int>(std::min<int64_t>((warps * 32 + kThreads - 1) / kThreads, 8LL * sms));
}

}  // namespace

void quant_fp8_rows(const void* x, void* codes, float* scales, int64_t rows, int hidden, cudaStream_t s) {
    if (rows <= 0) return;
    if (hidden <= 0 || hidden % 128) throw kiwi::error("quant_fp8_rows: hidden must be a positive multiple of 128");
    const int blocks = grid_for(rows * ((hidden + 511) / 512));
    quant_fp8_rows_kernel<<<blocks, kThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(x),
                                                      static_cast<uint8_t*>(codes), scales, rows, hidden);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

int nvfp4_scale_bytes(int hidden) { return (4 + hidden / 16 + 15) / 16 * 16; }

void quant_nvfp4_rows(const void* x, void* codes, void* scales, int64_t rows, int hidden, cudaStream_t s) {
    if (rows <= 0) return;
    if (hidden <= 0 || hidden % 16) throw kiwi::error("quant_nvfp4_rows: hidden must be a positive multiple of 16");
    const int blocks = grid_for(rows);
    quant_nvfp4_rows_kernel<<<blocks, kThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(x),
                                                        static_cast<uint8_t*>(codes), static_cast<uint8_t*>(scales),
                                                        rows, hidden, nvfp4_scale_bytes(hidden));
    KIWI_CUDA_CHECK(cudaGetLastError());
}

}  // namespace kiwi::ops
