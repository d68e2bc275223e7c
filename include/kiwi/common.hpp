// kiwi-b200: shared definitions for host and device code.
//
// Error handling on a shared GPU pool never traps: device code records an
// ErrorRecord in pinned host memory and returns a status; host code raises
// kiwi::error (a std::runtime_error) after it synchronises.
#pragma once

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>

#if defined(__CUDACC__)
#define KIWI_HD __host__ __device__ __forceinline__
#define KIWI_DEV __device__ __forceinline__
#else
#define KIWI_HD inline
#define KIWI_DEV inline
#endif

#define KIWI_VERSION_MAJOR 0
#define KIWI_VERSION_MINOR 1
#define KIWI_VERSION_PATCH 0

namespace kiwi {

class error : public std::runtime_error {
public:
    using std::runtime_error::runtime_error;
};

/// Status codes a device operation can return or record.
enum class Status : uint32_t {
    kOk = 0,
    kTimeout = 1,          // a bounded wait ran out
    kOversize = 2,         // message larger than the ring / kMaxMessageBytes
    kBadArgument = 3,      // index or size out of range (checked builds)
    kCorrupt = 4,          // a signal or header failed validation
    kPeerError = 5,        // a peer rank reported an error
};

inline const char* status_name(Status s) {
    switch (s) {
        case Status::kOk: return "ok";
        case Status::kTimeout: return "timeout";
        case Status::kOversize: return "oversize";
        case Status::kBadArgument: return "bad_argument";
        case Status::kCorrupt: return "corrupt";
        case Status::kPeerError: return "peer_error";
    }
    return "unknown";
}

/// One error record, written by device code into pinned host memory (or device
/// memory) with volatile stores.  `code` is written last so a host reader that
/// sees a non-zero code sees the other fields too (x86 TSO on the host side;
/// the device issues a system fence before the code store).
struct alignas(16) ErrorRecord {
    uint32_t code;   // Status, 0 = no error
    uint32_t site;   // call site id (see kiwi::site_*)
    uint32_t rank;   // reporting rank (or block id for single-GPU code)
    uint32_t info;   // site-specific detail (index, expected value, ...)
};

// Call-site ids recorded in ErrorRecord::site.
enum Site : uint32_t {
    site_none = 0,
    site_d2h_push = 1,
    site_d2h_mpsc_credit = 2,
    site_h2d_pop = 3,
    site_mpmc_pop = 4,
    site_reply_wait = 5,
    site_p2p_wait = 6,
    site_grid_barrier = 7,
    site_all2all_wait = 8,
    site_ep_flag_wait = 9,
    site_ep_capacity = 10,
    site_gemm_flag_wait = 11,
};

KIWI_HD constexpr bool is_pow2(uint64_t v) { return v != 0 && (v & (v - 1)) == 0; }

KIWI_HD constexpr uint32_t log2_pow2(uint64_t v) {
    uint32_t r = 0;
    while (v > 1) { v >>= 1; ++r; }
    return r;
}

KIWI_HD constexpr uint64_t round_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

}  // namespace kiwi

#define KIWI_CUDA_CHECK(expr)                                                        \
    do {                                                                             \
        cudaError_t kiwi_err_ = (expr);                                              \
        if (kiwi_err_ != cudaSuccess) {                                              \
            throw ::kiwi::error(std::string("CUDA error at ") + __FILE__ + ":" +     \
                                std::to_string(__LINE__) + " " #expr ": " +          \
                                cudaGetErrorString(kiwi_err_));                      \
        }                                                                            \
    } while (0)

#define KIWI_CU_CHECK(expr)                                                          \
    do {                                                                             \
        CUresult kiwi_res_ = (expr);                                                 \
        if (kiwi_res_ != CUDA_SUCCESS) {                                             \
            const char* kiwi_msg_ = nullptr;                                         \
            cuGetErrorString(kiwi_res_, &kiwi_msg_);                                 \
            throw ::kiwi::error(std::string("CUDA driver error at ") + __FILE__ +    \
                                ":" + std::to_string(__LINE__) + " " #expr ": " +    \
                                (kiwi_msg_ ? kiwi_msg_ : "?"));                      \
        }                                                                            \
    } while (0)
