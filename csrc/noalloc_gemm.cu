// Allocation-free C entry point of the grouped BF16 GEMM.
//
// This entry point has no counterpart in the reference (AMDResearch/kiwi has
// no GEMM at all); it is an addition of this library.
//
// Who needs it: callers that must not allocate device memory while they run.
// Typical cases are a serving engine that reserves all GPU memory for its own
// pool at start-up (any cudaMalloc later fails or fragments that pool), and C
// or C++ hosts that cannot reach PyTorch's caching allocator.  The regular entry point
// (kiwi_b200._C.ops.GroupedGemm) allocates its schedule buffers with torch;
// this one keeps them in a fixed device array instead.
//
// The contract (inputs, limits, the shared array, error codes) is stated in
// include/kiwi/gemm/noalloc.h, which declares the exported symbols.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "kiwi/gemm/grouped_gemm.hpp"
#include "kiwi/gemm/noalloc.h"

namespace {

constexpr int kNoallocMaxGroups = 1024;
constexpr int kScratchWords = 2 * (kNoallocMaxGroups + 1) + 64;  // offsets, tile prefix, error word (+ pad)
constexpr int kMaxDevices = 64;

static __device__ __align__(256) int32_t g_noalloc_scratch[kScratchWords];

std::mutex g_mu;
int32_t* g_scratch_ptr[kMaxDevices] = {};
thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

/// Device address of this device's copy of the scratch array (resolved once per device).
int32_t* scratch_for_current_device(std::string& err) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        err = std::string("cudaGetDevice failed: ") + cudaGetErrorString(e);
        return nullptr;
    }
    if (dev < 0 || dev >= kMaxDevices) {
        err = "device index beyond the supported 64 devices";
        return nullptr;
    }
    std::lock_guard<std::mutex> g(g_mu);
    if (g_scratch_ptr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) {
            err = std::string("cudaGetSymbolAddress(scratch) failed: ") + cudaGetErrorString(e);
            return nullptr;
        }
        g_scratch_ptr[dev] = static_cast<int32_t*>(p);
    }
    return g_scratch_ptr[dev];
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" __attribute__((visibility("default"))) int kiwi_noalloc_max_groups(void) { return kNoallocMaxGroups; }

extern "C" __attribute__((visibility("default"))) const char* kiwi_noalloc_last_error(void) {
    return g_last_error.c_str();
}

/// C[g rows] = A[g rows] . B[g]^T per group g (optionally SwiGLU and a per-row
/// scale in the epilogue), without allocating.  See the file comment.
extern "C" __attribute__((visibility("default"))) int kiwi_grouped_gemm_bf16_noalloc(
    const void* a, int64_t a_rows, const void* b, int32_t num_groups, int32_t n, int32_t k, const int32_t* counts,
    void* c, int64_t c_rows, int32_t swiglu, const float* row_scale, void* stream) {
    g_last_error.clear();
    if (num_groups < 1 || num_groups > kNoallocMaxGroups) {
        return fail(1, "kiwi_grouped_gemm_bf16_noalloc: num_groups must be in [1, " +
                           std::to_string(kNoallocMaxGroups) + "], got " + std::to_string(num_groups));
    }
    if (n <= 0 || n % 256 != 0 || k <= 0 || k % 64 != 0) {
        return fail(2, "kiwi_grouped_gemm_bf16_noalloc: n must be a positive multiple of 256 and k of 64");
    }
    if (!a || !b || !c || !counts || a_rows <= 0 || c_rows <= 0) {
        return fail(3, "kiwi_grouped_gemm_bf16_noalloc: null pointer or empty A/C");
    }
    if (!aligned16(a) || !aligned16(b) || !aligned16(c)) {
        return fail(4, "kiwi_grouped_gemm_bf16_noalloc: A, B and C must be 16-byte aligned");
    }
    std::string err;
    int32_t* scratch = scratch_for_current_device(err);
    if (!scratch) return fail(5, "kiwi_grouped_gemm_bf16_noalloc: " + err);
    int32_t* offsets = scratch;
    int32_t* tiles = scratch + (kNoallocMaxGroups + 1);
    int32_t* error_word = scratch + 2 * (kNoallocMaxGroups + 1);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    try {
        const cudaError_t e = cudaMemsetAsync(error_word, 0, sizeof(int32_t), s);
        if (e != cudaSuccess) return fail(6, std::string("cudaMemsetAsync failed: ") + cudaGetErrorString(e));
        const CUtensorMap tmap_a = kiwi::gemm::make_tmap_bf16_2d(a, static_cast<uint64_t>(a_rows), k, 128);
        const CUtensorMap tmap_b =
            kiwi::gemm::make_tmap_bf16_2d(b, static_cast<uint64_t>(num_groups) * n, k, 256);
        kiwi::gemm::build_schedule(counts, num_groups, n, 256, offsets, tiles, s);
        kiwi::gemm::GroupedArgs args{};
        args.m64_tails = 1;
        args.group_offset = offsets;
        args.tile_prefix = tiles;
        args.num_groups = num_groups;
        args.n = n;
        args.k = k;
        args.c = static_cast<__nv_bfloat16*>(c);
        args.ldc = swiglu ? n / 2 : n;
        args.row_scale = row_scale;
        args.error = reinterpret_cast<uint32_t*>(error_word);
        args.max_rows = c_rows;
        kiwi::gemm::grouped_gemm(tmap_a, tmap_b, args, swiglu != 0, 0, s);
    } catch (const std::exception& ex) {
        return fail(7, std::string("kiwi_grouped_gemm_bf16_noalloc: ") + ex.what());
    }
    return 0;
}

/// Copies this device's error word to caller memory and synchronises `stream`
/// (see noalloc.h).  Allocates nothing.
extern "C" __attribute__((visibility("default"))) int kiwi_noalloc_error_word(int32_t* host_out, void* stream) {
    g_last_error.clear();
    if (!host_out) return fail(3, "kiwi_noalloc_error_word: null host_out");
    std::string err;
    int32_t* scratch = scratch_for_current_device(err);
    if (!scratch) return fail(5, "kiwi_noalloc_error_word: " + err);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(host_out, scratch + 2 * (kNoallocMaxGroups + 1), sizeof(int32_t),
                                    cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return fail(6, std::string("kiwi_noalloc_error_word: ") + cudaGetErrorString(e));
    return 0;
}
