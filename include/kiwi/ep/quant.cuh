// kiwi::ep element formats on the device: bf16 <-> fp32 packing, 1x128
// block-scaled FP8 e4m3 and NVFP4 (e2m1 with e4m3 scales per 16 elements
// relative to an fp32 row scale) quantisation of 16-element lane chunks.
// Shared by the dispatch / receive kernels and the grouped GEMM's gathering
// A producer, so every path rounds identically.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp4.h>
#include <cuda_fp8.h>

#include "kiwi/common.hpp"

namespace kiwi::ep {

inline constexpr float kFp8Max = 448.0f;
inline constexpr float kFp4Max = 6.0f;

#if defined(__CUDACC__)

KIWI_DEV void bf16x8_to_f32(uint4 u, float (&f)[8]) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 t = __bfloat1622float2(h[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

KIWI_DEV uint4 f32x8_to_bf16(const float (&f)[8]) {
    uint4 u;
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
        w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    return u;
}

/// FP8 1x128: lane covers 16 elements of a 512-element chunk; 8 lanes share a block scale.
KIWI_DEV void quant_fp8_16(const uint4 (&in)[2], float& scale, uint4& out) {
    float f[16];
    float a[8];
    bf16x8_to_f32(in[0], a);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = a[i];
    bf16x8_to_f32(in[1], a);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[8 + i] = a[i];
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(f[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
    scale = amax > 0.f ? amax / kFp8Max : 1.0f;
    const float inv = amax > 0.f ? kFp8Max / amax : 0.f;
    uint16_t q[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        q[i] = __nv_cvt_float2_to_fp8x2(make_float2(f[2 * i] * inv, f[2 * i + 1] * inv), __NV_SATFINITE, __NV_E4M3);
    }
    out = make_uint4(q[0] | (uint32_t(q[1]) << 16), q[2] | (uint32_t(q[3]) << 16), q[4] | (uint32_t(q[5]) << 16),
                     q[6] | (uint32_t(q[7]) << 16));
}

KIWI_DEV void dequant_fp8_16(uint4 q, float scale, uint4 (&out)[2]) {
    const uint16_t* p = reinterpret_cast<const uint16_t*>(&q);
    float f[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(p[i]), __NV_E4M3);
        const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&hr));
        f[2 * i] = t.x * scale;
        f[2 * i + 1] = t.y * scale;
    }
    float a[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = f[i];
    out[0] = f32x8_to_bf16(a);
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = f[8 + i];
    out[1] = f32x8_to_bf16(a);
}

/// NVFP4: lane covers 16 elements = one 16-element block (e4m3 block scale,
/// relative to a per-row fp32 scale so block scales stay in e4m3 range).
KIWI_DEV void quant_fp4_16(const uint4 (&in)[2], float row_scale, uint8_t& sbyte, uint2& out) {
    float f[16];
    float a[8];
    bf16x8_to_f32(in[0], a);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = a[i];
    bf16x8_to_f32(in[1], a);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[8 + i] = a[i];
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(f[i]));
    // block scale in e4m3 units of row_scale: s = amax / (6 * row_scale)
    const float s = row_scale > 0.f ? amax / (kFp4Max * row_scale) : 0.f;
    const __nv_fp8_storage_t sq = __nv_cvt_float_to_fp8(s, __NV_SATFINITE, __NV_E4M3);
    const __half_raw sh = __nv_cvt_fp8_to_halfraw(sq, __NV_E4M3);
    const float sdec = __half2float(*reinterpret_cast<const __half*>(&sh)) * row_scale;
    const float inv = sdec > 0.f ? 1.0f / sdec : 0.f;
    sbyte = sq;
    uint8_t b[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        b[i] = __nv_cvt_float2_to_fp4x2(make_float2(f[2 * i] * inv, f[2 * i + 1] * inv), __NV_E2M1, cudaRoundNearest);
    }
    out = make_uint2(b[0] | (uint32_t(b[1]) << 8) | (uint32_t(b[2]) << 16) | (uint32_t(b[3]) << 24),
                     b[4] | (uint32_t(b[5]) << 8) | (uint32_t(b[6]) << 16) | (uint32_t(b[7]) << 24));
}

KIWI_DEV void dequant_fp4_16(uint2 q, float block_scale, uint4 (&out)[2]) {
    const uint8_t* p = reinterpret_cast<const uint8_t*>(&q);
    float f[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const __half2_raw hr = __nv_cvt_fp4x2_to_halfraw2(static_cast<__nv_fp4x2_storage_t>(p[i]), __NV_E2M1);
        const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&hr));
        f[2 * i] = t.x * block_scale;
        f[2 * i + 1] = t.y * block_scale;
    }
    float a[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = f[i];
    out[0] = f32x8_to_bf16(a);
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = f[8 + i];
    out[1] = f32x8_to_bf16(a);
}

#endif  // __CUDACC__

}  // namespace kiwi::ep
