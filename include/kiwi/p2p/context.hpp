// kiwi::p2p::Context: symmetric heap + invoke control plane + proxy threads.
//
// Parity with the reference's context_t / gcontext_t / ghandle_t
// (apps/p2p/context.hip.{hpp,cpp} of AMDResearch/kiwi): num_queues invoke
// endpoints, proxy threads pinned to GPU-local cores that run built-in and
// user callbacks, a by-value device context, a move-only device handle that
// saves its queue position when it goes out of scope.  The reference's data
// path (proxy -> LCI RDMA put + readiness byte) becomes, on B200:
//   * put / get / signal / wait issued by the kernel itself over NVLink
//     (include/kiwi/p2p/device.cuh) -- the fast path;
//   * post_ce_put: the kernel posts a descriptor; a proxy thread issues a
//     copy-engine cudaMemcpyAsync into the peer's heap, then writes the
//     peer's flag and the local completion counter in stream order
//     (cuStreamWriteValue64) -- for bulk copies that should not occupy SMs,
//     the counterpart of the reference's SDMA ping-pong example;
//   * host_signal: a proxy thread stores a value into any rank's flag.
#pragma once

#include <cuda_runtime.h>

#include <memory>
#include <vector>

#include "kiwi/invoke/invoke.hpp"
#include "kiwi/invoke/progress.hpp"
#include "kiwi/p2p/heap.hpp"

namespace kiwi::p2p {

/// Copy-engine put: heap[dst_rank][dst_off, +bytes) = local heap[src_off, +bytes),
/// then heap[flag_rank][flag_off] = flag_value and the local completion counter
/// (`counter_off` in the local heap) = counter_value, both in stream order.
struct alignas(8) CePutDesc {
    uint32_t dst_rank;
    uint32_t flag_rank;
    uint64_t dst_off;
    uint64_t src_off;
    uint64_t bytes;
    uint64_t flag_off;
    uint64_t flag_value;
    uint64_t counter_off;
    uint64_t counter_value;
};

/// Host-executed store of `value` into heap[rank][off] (8 bytes).
struct alignas(8) HostSignalDesc {
    uint32_t rank;
    uint32_t pad;
    uint64_t off;
    uint64_t value;
};

using ControlQueue = queue::SPSCD2HQueue;

/// By-value device context of a Context.
struct GContext {
    HeapView heap;
    invoke::DeviceContext<ControlQueue>* invoke;
    uint8_t ce_put_cb;
    uint8_t host_signal_cb;
    uint8_t pad[6];
};

class Context {
public:
    Context(SymmetricHeap& heap, size_t num_queues, uint64_t queue_capacity = 2048);
    ~Context();
    Context(const Context&) = delete;
    Context& operator=(const Context&) = delete;

    /// User callbacks on the control plane (ids shared by every queue).
    template <typename... Args>
    uint8_t register_callback(std::function<void(Args...)> fn) {
        return ictx_->register_callback(std::move(fn));
    }
    uint8_t register_raw_callback(invoke::RawCallback::Fn fn, uint32_t bytes) {
        return ictx_->register_raw_callback(std::move(fn), bytes);
    }

    /// Starts `n` proxy threads pinned to `cpus` (GPU-local cores if empty).
    void spawn_proxy_threads(size_t n, std::vector<int> cpus = {});
    /// Drains and joins the proxy threads, then waits for issued copies.
    void join_proxy_threads();

    GContext device_context() const;
    invoke::Context<ControlQueue>& invoke_context() { return *ictx_; }
    SymmetricHeap& heap() { return heap_; }
    uint64_t copies_issued() const { return copies_; }
    /// Proxy-thread totals (callbacks = control messages served).
    invoke::ProgressStats proxy_stats() const { return threads_->stats(); }
    /// Proxy threads serve only queues [0, n) (0 = all); a shrink drains the
    /// dropped queues once (invoke::ProgressThreads::set_active_endpoints).
    uint32_t set_active_queues(size_t n) { return threads_->set_active_endpoints(n); }
    bool active_applied(uint32_t generation) const { return threads_->active_applied(generation); }

private:
    void ce_put(const CePutDesc& d);
    void host_signal(const HostSignalDesc& d);

    SymmetricHeap& heap_;
    int device_;
    std::unique_ptr<invoke::Context<ControlQueue>> ictx_;
    std::unique_ptr<invoke::ProgressThreads<ControlQueue>> threads_;
    cudaStream_t ce_stream_ = nullptr;
    uint8_t ce_put_cb_ = 0, host_signal_cb_ = 0;
    std::atomic<uint64_t> copies_{0};
    std::mutex ce_mu_;
};

}  // namespace kiwi::p2p
