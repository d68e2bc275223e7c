// kiwi::p2p symmetric heap over NVLink 5 / NVSwitch.
//
// Parity: the reference registers a buffer with LCI on every rank and
// all-gathers remote keys (register_symmetric, apps/p2p/context.hip.cpp:174-210
// of AMDResearch/kiwi) and, for same-node peers, opens HIP IPC handles
// (apps/ep/ep_context.hip.cpp:375-460).  On B200 every peer is one NVSwitch hop
// away, so the heap is device memory every rank maps directly:
//   cuMemCreate (POSIX-FD shareable) -> export FD -> exchange FDs over
//   abstract Unix sockets (SCM_RIGHTS) -> cuMemImportFromShareableHandle ->
//   cuMemMap + cuMemSetAccess into one local VA range per peer.
// Optionally an NVLS multicast object is bound over every rank's heap so
// multimem.st / multimem.ld_reduce reach all ranks with one instruction.
#pragma once

#include <cuda.h>

#include <functional>
#include <string>
#include <vector>

#include "kiwi/common.hpp"

namespace kiwi::p2p {

inline constexpr int kMaxRanks = 16;

/// Device-copyable view of a heap: pass by value to kernels.
struct HeapView {
    uint8_t* base[kMaxRanks];  // base[r] = rank r's heap mapped in this process
    uint8_t* mc;               // NVLS multicast mapping (nullptr when disabled)
    uint64_t size;
    int32_t rank;
    int32_t world;
    // Checked mode (null: off).  Every put / get / signal of the device API
    // validates (rank, offset, bytes) against [0, check_limit); the first bad
    // access is recorded as check[0..3] = {1, site, rank, offset low 32 bits}
    // and every bad access is skipped instead of touching memory.
    uint32_t* check;
    uint64_t check_limit;
};

/// Sites recorded by the checked mode (HeapView::check[1]).
enum CheckSite : uint32_t {
    kCheckPut = 1,
    kCheckGet = 2,
    kCheckSignal = 3,
    kCheckLl8 = 4,
    kCheckMulticast = 5,
};

/// True when [off, off + bytes) of rank's heap lies inside [0, limit).
KIWI_HD constexpr bool heap_range_ok(int world, uint64_t limit, int rank, uint64_t off, uint64_t bytes) {
    return rank >= 0 && rank < world && off <= limit && bytes <= limit - off;
}

/// Exchanges one file descriptor per rank through abstract Unix sockets named
/// "kiwi.<job>.<rank>".  Returns fds[r] = a descriptor for rank r's object in
/// this process (fds[rank] is a dup of `my_fd`).  All ranks call it together.
std::vector<int> exchange_fds(const std::string& job, int rank, int world, int my_fd,
                              double timeout_s = 60.0);

/// Root sends `fd` to every other rank; returns this process's descriptor.
int broadcast_fd(const std::string& job, int rank, int world, int root, int fd,
                 double timeout_s = 60.0);

class SymmetricHeap {
public:
    using Barrier = std::function<void()>;

    /// Collective.  `bytes` is rounded up to the allocation granularity.
    /// `barrier` must be a host barrier over the same ranks (used by the
    /// multicast set-up between AddDevice and BindMem).
    SymmetricHeap(int device, size_t bytes, int rank, int world, const std::string& job,
                  bool multicast, Barrier barrier);
    ~SymmetricHeap();
    SymmetricHeap(const SymmetricHeap&) = delete;
    SymmetricHeap& operator=(const SymmetricHeap&) = delete;

    void* local() const { return view_.base[view_.rank]; }
    void* peer(int r) const { return view_.base[r]; }
    void* multicast() const { return view_.mc; }
    size_t size() const { return view_.size; }
    int rank() const { return view_.rank; }
    int world() const { return view_.world; }
    const HeapView& view() const { return view_; }
    /// Checked mode: `record` = 4 device uint32 words (null: off); accesses
    /// must stay below `limit` (0 or more than the size: the whole heap).
    void set_checks(uint32_t* record, uint64_t limit) {
        view_.check = record;
        view_.check_limit = (limit == 0 || limit > view_.size) ? view_.size : limit;
    }

    /// True when the device supports NVLS multicast objects.
    static bool multicast_supported(int device);

private:
    void map_range(CUmemGenericAllocationHandle h, void** va);
    void release() noexcept;

    int device_;
    HeapView view_{};
    CUmemGenericAllocationHandle local_handle_ = 0;
    std::vector<CUmemGenericAllocationHandle> handles_;  // per rank (local included)
    CUmemGenericAllocationHandle mc_handle_ = 0;
    bool mc_bound_ = false;
    size_t granularity_ = 0;
};

}  // namespace kiwi::p2p
