// Host API of the row-copy kernels (csrc/rows_gpu.cu): the EP pack, unpack and
// accumulate patterns as stand-alone kernels, for copy-bandwidth measurements
// against the HBM roofline.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace kiwi::ops {

// Error bits the kernels OR into their error word (nothing is written for a
// row whose index is out of range; negative indices mean "no row" and are
// skipped without an error).
constexpr uint32_t kRowsSrcRange = 1u;  // a source index >= src_rows
constexpr uint32_t kRowsDstRange = 2u;  // a destination index >= dst_rows
constexpr int kRowsMaxK = 64;           // rows summed per output row, at most

/// dst[dst_idx ? dst_idx[i] : i] = src[src_idx ? src_idx[i] : i] for i < rows;
/// rows of row_bytes bytes (a multiple of 16; both base pointers 16-byte
/// aligned).  grid <= 0: four CTAs per SM.
void rows_copy(const void* src, void* dst, const int32_t* src_idx, const int32_t* dst_idx, int64_t rows,
               int64_t row_bytes, int64_t src_rows, int64_t dst_rows, uint32_t* error, int grid, cudaStream_t s);

/// out[t] = sum over j < k of src[map[t * k + j]] (bf16 rows of `hidden`
/// elements, a multiple of 8; fp32 sums, round-to-nearest bf16 out); entries
/// < 0 are skipped, a token with none gets zeros.  k <= kRowsMaxK.
void rows_accumulate_bf16(const void* src, void* out, const int32_t* map, int64_t tokens, int k, int64_t hidden,
                          int64_t src_rows, uint32_t* error, int grid, cudaStream_t s);

}  // namespace kiwi::ops
