// Host API of the stand-alone FP8 quantisation kernel (csrc/quant_gpu.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace kiwi::ops {

/// 1x128 block FP8 e4m3 quantisation of bf16 rows x [rows, hidden] (hidden a
/// multiple of 128, x 16-byte aligned): codes [rows, hidden] (e4m3 bytes) and
/// fp32 scales [rows, hidden / 128] with scale = amax / 448 (1 for an all-zero
/// block).  The arithmetic is the EP dispatch kernel's (kiwi/ep/quant.cuh).
void quant_fp8_rows(const void* x, void* codes, float* scales, int64_t rows, int hidden, cudaStream_t s);

}  // namespace kiwi::ops
