// kiwi::p2p completion counter: host threads signal, kernels poll.
//
// Parity with the reference's comp_counter_t (apps/p2p/comp_counter.hip.hpp:15-86
// of AMDResearch/kiwi: a counter in managed memory that the CPU bumps with
// fetch_add when a proxied operation completes and GPU code reads, sets or
// polls).  Here the counter is one 64-bit word in mapped pinned host memory
// (cudaHostAlloc Mapped|Portable): the host bumps it with a release
// fetch_add; the device reads it with ld.acquire.sys and polls under a
// deadline, so a signal that never comes returns kTimeout instead of hanging.
#pragma once

#include <atomic>
#include <cstdint>

#include "kiwi/common.hpp"
#include "kiwi/queue/host_memory.hpp"
#if defined(__CUDACC__)
#include "kiwi/ptx.cuh"
#endif

namespace kiwi::p2p {

/// By-value device view of a CompletionCounter.
struct CounterView {
    uint64_t* word;  // device-visible address

#if defined(__CUDACC__)
    KIWI_DEV uint64_t get() const { return ptx::ld_acquire_sys_u64(word); }
    KIWI_DEV void set(uint64_t v) const { ptx::st_release_sys_u64(word, v); }
    KIWI_DEV void add(uint64_t v) const { ptx::red_release_sys_add_u64(word, v); }
    /// One thread: waits until the counter reaches `want` (>=), or the
    /// deadline passes.
    KIWI_DEV Status poll(uint64_t want, uint64_t timeout_ns) const {
        if (get() >= want) return Status::kOk;
        ptx::Deadline dl(timeout_ns);
        while (get() < want) {
            if (dl.expired()) return Status::kTimeout;
        }
        return Status::kOk;
    }
#endif
};

/// Host side: owns the word.  Without a GPU it lives in plain host memory
/// (host-only tests).
class CompletionCounter {
public:
    explicit CompletionCounter(queue::MemKind kind = queue::default_host_kind())
        : kind_(kind), mem_(queue::alloc_zeroed(64, kind)) {}
    ~CompletionCounter() { queue::free_memory(mem_, kind_); }
    CompletionCounter(const CompletionCounter&) = delete;
    CompletionCounter& operator=(const CompletionCounter&) = delete;

    /// Adds `n` (release) and returns the new value.
    uint64_t signal(uint64_t n = 1) { return __atomic_add_fetch(word(), n, __ATOMIC_RELEASE); }
    uint64_t get() const { return __atomic_load_n(word(), __ATOMIC_ACQUIRE); }
    void set(uint64_t v) { __atomic_store_n(word(), v, __ATOMIC_RELEASE); }
    CounterView device_view() const {
        return CounterView{static_cast<uint64_t*>(queue::device_address(mem_, kind_))};
    }

private:
    uint64_t* word() const { return static_cast<uint64_t*>(mem_); }
    queue::MemKind kind_;
    void* mem_;
};

}  // namespace kiwi::p2p
