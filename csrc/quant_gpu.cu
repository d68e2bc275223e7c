// Stand-alone 1x128 FP8 quantisation of bf16 rows with the EP dispatch
// kernel's arithmetic (kiwi/ep/quant.cuh: quant_fp8_16), for callers that
// quantise outside the fused dispatch, such as the all-to-all EP transport.
// One warp per 512-element chunk of a row: each lane converts 16 elements and
// eight lanes share one block scale.
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

}  // namespace

void quant_fp8_rows(const void* x, void* codes, float* scales, int64_t rows, int hidden, cudaStream_t s) {
    if (rows <= 0) return;
    if (hidden <= 0 || hidden % 128) throw kiwi::error("quant_fp8_rows: hidden must be a positive multiple of 128");
    int dev = 0, sms = 0;
    KIWI_CUDA_CHECK(cudaGetDevice(&dev));
    KIWI_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int64_t warps = rows * ((hidden + 511) / 512);
    const int64_t blocks = std::min<int64_t>((warps * 32 + kThreads - 1) / kThreads, 8LL * sms);
    quant_fp8_rows_kernel<<<static_cast<int>(blocks), kThreads, 0, s>>>(
        static_cast<const __nv_bfloat16*>(x), static_cast<uint8_t*>(codes), scales, rows, hidden);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

}  // namespace kiwi::ops
