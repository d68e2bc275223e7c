/* Allocation-free C entry point of the grouped BF16 GEMM (csrc/noalloc_gemm.cu,
 * exported from the kiwi_b200 extension library).
 *
 * This entry point has no counterpart in the reference (AMDResearch/kiwi has no
 * GEMM); it is an addition of this library.
 *
 * It is meant for callers that must not allocate device memory once they run:
 * a serving engine that reserved the whole GPU for its own pool at start-up
 * (a later cudaMalloc fails or fragments that pool), or a C / C++ host that
 * has no PyTorch caching allocator to draw from.  The regular entry point
 * (kiwi_b200._C.ops.GroupedGemm) allocates its schedule with torch; this one
 * keeps its scratch (group offsets, tile prefix, error word) in one fixed
 * device array compiled into the library.
 *
 * Contract:
 *   - The caller passes every input and output: A [a_rows, k] bf16, B
 *     [num_groups * n, k] bf16 (both row-major, 16-byte aligned), counts
 *     int32[num_groups] (device memory, rows per group; group g's rows follow
 *     group g-1's in A and C), C [c_rows, n] bf16 ([c_rows, n / 2] with
 *     swiglu), an optional fp32 row_scale with at least c_rows entries (device
 *     memory; NULL for none), and the CUDA stream (NULL = legacy default).
 *     Rows at or past c_rows are neither written nor scaled.
 *   - At most kiwi_noalloc_max_groups() (1024) groups; larger requests are
 *     rejected.  The array takes 8.5 KB on every GPU that loads the library,
 *     until the process exits.
 *   - The first call on a device (with that device current) looks up the
 *     array's device address with cudaGetSymbolAddress and caches it; make
 *     that first call before any stream capture.
 *   - All calls share the array, which keeps the last call's contents; each
 *     call clears the error word and rewrites the schedule.  Calls that
 *     overlap on one GPU (two streams, two host threads) race on the array and
 *     must be serialised; calls on different GPUs use different copies.
 *   - No cudaMalloc, cudaFree or allocating library routine is called.
 *   - Return value 0 on success; otherwise a non-zero code, with a message
 *     from kiwi_noalloc_last_error() (per host thread): 1 group count, 2 n / k
 *     shape, 3 null pointer or empty A / C, 4 alignment, 5 device set-up,
 *     6 CUDA call, 7 launch.
 *   - The kernel runs asynchronously.  A bounded wait inside it that ran out
 *     (the kernel then stops early and C is incomplete) is recorded in the
 *     error word; read it with kiwi_noalloc_error_word() after the call's work
 *     on the stream is done and before the next call, which clears it.
 */
#ifndef KIWI_GEMM_NOALLOC_H
#define KIWI_GEMM_NOALLOC_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/** Largest num_groups the allocation-free entry accepts (1024). */
int kiwi_noalloc_max_groups(void);

/** Message of the last failed call on this host thread ("" after a success). */
const char* kiwi_noalloc_last_error(void);

/** C[rows of group g] = A[rows of group g] . B[g]^T, times row_scale[row].
 *  With swiglu != 0, B[g]'s n rows are blocks of 128 gate rows followed by the
 *  128 matching up rows, and C gets silu(gate) * up, n / 2 columns.  See the
 *  contract above. */
int kiwi_grouped_gemm_bf16_noalloc(const void* a, int64_t a_rows, const void* b, int32_t num_groups, int32_t n,
                                   int32_t k, const int32_t* counts, void* c, int64_t c_rows, int32_t swiglu,
                                   const float* row_scale, void* stream);

/** Copies the current device's error word into *host_out (pageable or pinned
 *  host memory) on `stream` and synchronises the stream.  0 = the last call's
 *  kernel ran to completion; non-zero = one of its bounded waits ran out.
 *  Returns 0, or 3 (null host_out), 5 (device set-up) or 6 (CUDA call). */
int kiwi_noalloc_error_word(int32_t* host_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KIWI_GEMM_NOALLOC_H */
