// Host API of the stand-alone quantisation kernels (csrc/quant_gpu.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace kiwi::ops {

/// 1x128 block FP8 e4m3 quantisation of bf16 rows x [rows, hidden] (hidden a
/// multiple of 128, x 16-byte aligned): codes [rows, hidden] (e4m3 bytes) and
/// fp32 scales [rows, hidden / 128] with scale = amax / 448 (1 for an all-zero
/// block).  The arithmetic is the EP dispatch kernel's (kiwi/ep/quant.cuh).
void quant_fp8_rows(const void* x, void* codes, float* scales, int64_t rows, int hidden, cudaStream_t s);

/// Scale bytes of one NVFP4 row: fp32 row scale, one e4m3 byte per 16
/// elements, zero padding to a multiple of 16 bytes.
int nvfp4_scale_bytes(int hidden);

/// NVFP4 quantisation of bf16 rows x [rows, hidden] (hidden a multiple of 16,
/// x 16-byte aligned) into the NVLink dispatch's wire bytes: packed e2m1 codes
/// [rows, hidden / 2] (element 2i in the low nibble) and scale bytes
/// [rows, nvfp4_scale_bytes(hidden)] (fp32 row scale amax / (448 * 6), then
/// the e4m3 block scales relative to it).  Bit-identical to the dispatch
/// kernel's quantisation of the same row.
void quant_nvfp4_rows(const void* x, void* codes, void* scales, int64_t rows, int hidden, cudaStream_t s);

}  // namespace kiwi::ops
