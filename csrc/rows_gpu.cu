// Row-copy kernels: the pack (gather), unpack (scatter), plain copy and
// accumulate (top-k sum) patterns of EP dispatch and combine, on their own.
//
// They are the counterparts of the reference's copy microbenchmarks
// (apps/ep/benchmarks/bench_ep_copy.hip.cpp, bench_ep_hidden_copy.hip.cpp of
// AMDResearch/kiwi: pack / unpack / accumulate hidden-copy kernels) and give
// the HBM side of the EP roofline: what a row-granular copy reaches on B200
// when nothing else runs.  One CTA per row at a time (grid-stride over rows),
// 16-byte vector accesses, four vectors in flight per thread.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "kiwi/common.hpp"
#include "kiwi/ops/rows.hpp"

namespace kiwi::ops {

namespace {

constexpr int kThreads = 128;

__global__ void __launch_bounds__(kThreads) rows_copy_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                                              const int32_t* __restrict__ src_idx,
                                                              const int32_t* __restrict__ dst_idx, int64_t rows,
                                                              int32_t vecs, int64_t src_rows, int64_t dst_rows,
                                                              uint32_t* error) {
    for (int64_t i = blockIdx.x; i < rows; i += gridDim.x) {
        const int64_t s = src_idx ? static_cast<int64_t>(src_idx[i]) : i;
        const int64_t d = dst_idx ? static_cast<int64_t>(dst_idx[i]) : i;
        if (s < 0 || d < 0) continue;
        if (s >= src_rows || d >= dst_rows) {
            if (threadIdx.x == 0) atomicOr(error, (s >= src_rows ? kRowsSrcRange : 0u) | (d >= dst_rows ? kRowsDstRange : 0u));
            continue;
        }
        const uint4* sp = src + s * vecs;
        uint4* dp = dst + d * vecs;
        int v = threadIdx.x;
        for (; v + 3 * kThreads < vecs; v += 4 * kThreads) {
            const uint4 a = __ldg(sp + v);
            const uint4 b = __ldg(sp + v + kThreads);
            const uint4 c = __ldg(sp + v + 2 * kThreads);
            const uint4 e = __ldg(sp + v + 3 * kThreads);
            dp[v] = a;
            dp[v + kThreads] = b;
            dp[v + 2 * kThreads] = c;
            dp[v + 3 * kThreads] = e;
        }
        for (; v < vecs; v += kThreads) dp[v] = __ldg(sp + v);
    }
}

__device__ __forceinline__ void add_bf16x8(float (&acc)[8], const uint4& x) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&x);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        acc[2 * i] += f.x;
        acc[2 * i + 1] += f.y;
    }
}

__global__ void __launch_bounds__(kThreads) rows_accumulate_kernel(const uint4* __restrict__ src,
                                                                    uint4* __restrict__ out,
                                                                    const int32_t* __restrict__ map, int64_t tokens,
                                                                    int k, int32_t vecs, int64_t src_rows,
                                                                    uint32_t* error) {
    __shared__ int64_t rows_s[kRowsMaxK];
    __shared__ int n_s;
    for (int64_t t = blockIdx.x; t < tokens; t += gridDim.x) {
        if (threadIdx.x == 0) {
            int n = 0;
            for (int j = 0; j < k; ++j) {
                const int64_t r = map[t * k + j];
                if (r < 0) continue;
                if (r >= src_rows) {
                    atomicOr(error, kRowsSrcRange);
                    continue;
                }
                rows_s[n++] = r;
            }
            n_s = n;
        }
        __syncthreads();
        const int n = n_s;
        for (int v = threadIdx.x; v < vecs; v += kThreads) {
            float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            int j = 0;
            for (; j + 1 < n; j += 2) {  // two rows in flight
                const uint4 a = __ldg(src + rows_s[j] * vecs + v);
                const uint4 b = __ldg(src + rows_s[j + 1] * vecs + v);
                add_bf16x8(acc, a);
                add_bf16x8(acc, b);
            }
            if (j < n) add_bf16x8(acc, __ldg(src + rows_s[j] * vecs + v));
            uint4 o;
            __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
            for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
            out[t * vecs + v] = o;
        }
        __syncthreads();  // rows_s is rewritten for the next token
    }
}

int default_grid(int64_t rows, int grid) {
    if (grid > 0) return grid;
    int dev = 0, sms = 0;
    KIWI_CUDA_CHECK(cudaGetDevice(&dev));
    KIWI_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int64_t g = 4LL * sms;
    return static_cast<int>(rows < g ? (rows > 0 ? rows : 1) : g);
}

}  // namespace

void rows_copy(const void* src, void* dst, const int32_t* src_idx, const int32_t* dst_idx, int64_t rows,
               int64_t row_bytes, int64_t src_rows, int64_t dst_rows, uint32_t* error, int grid, cudaStream_t s) {
    if (rows <= 0) return;
    rows_copy_kernel<<<default_grid(rows, grid), kThreads, 0, s>>>(
        static_cast<const uint4*>(src), static_cast<uint4*>(dst), src_idx, dst_idx, rows,
        static_cast<int32_t>(row_bytes / 16), src_rows, dst_rows, error);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

void rows_accumulate_bf16(const void* src, void* out, const int32_t* map, int64_t tokens, int k, int64_t hidden,
                          int64_t src_rows, uint32_t* error, int grid, cudaStream_t s) {
    if (tokens <= 0) return;
    rows_accumulate_kernel<<<default_grid(tokens, grid), kThreads, 0, s>>>(
        static_cast<const uint4*>(src), static_cast<uint4*>(out), map, tokens, k, static_cast<int32_t>(hidden / 8),
        src_rows, error);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

}  // namespace kiwi::ops
