#include "kiwi/p2p/context.hpp"

#include "kiwi/p2p/driver.hpp"
#include "kiwi/topology.hpp"

namespace kiwi::p2p {

Context::Context(SymmetricHeap& heap, size_t num_queues, uint64_t queue_capacity) : heap_(heap) {
    KIWI_CUDA_CHECK(cudaGetDevice(&device_));
    ictx_ = std::make_unique<invoke::Context<ControlQueue>>(num_queues, queue_capacity);
    threads_ = std::make_unique<invoke::ProgressThreads<ControlQueue>>(*ictx_);
    KIWI_CUDA_CHECK(cudaStreamCreateWithFlags(&ce_stream_, cudaStreamNonBlocking));
    ce_put_cb_ = ictx_->register_callback(std::function<void(CePutDesc)>([this](CePutDesc d) { ce_put(d); }));
    host_signal_cb_ =
        ictx_->register_callback(std::function<void(HostSignalDesc)>([this](HostSignalDesc d) { host_signal(d); }));
}

Context::~Context() {
    try {
        join_proxy_threads();
    } catch (...) {
    }
    if (ce_stream_) cudaStreamDestroy(ce_stream_);
}

void Context::ce_put(const CePutDesc& d) {
    const HeapView& v = heap_.view();
    if (d.dst_rank >= static_cast<uint32_t>(v.world) || d.flag_rank >= static_cast<uint32_t>(v.world) ||
        d.dst_off + d.bytes > v.size || d.src_off + d.bytes > v.size || d.flag_off + 8 > v.size ||
        d.counter_off + 8 > v.size) {
        throw kiwi::error("kiwi::p2p: copy-engine put descriptor out of the heap's range");
    }
    std::lock_guard<std::mutex> g(ce_mu_);
    KIWI_CUDA_CHECK(cudaSetDevice(device_));
    if (d.bytes) {
        KIWI_CUDA_CHECK(cudaMemcpyAsync(v.base[d.dst_rank] + d.dst_off, v.base[v.rank] + d.src_off, d.bytes,
                                        cudaMemcpyDeviceToDevice, ce_stream_));
    }
    const Driver& drv = driver();
    check_cu(drv.cuStreamWriteValue64(reinterpret_cast<CUstream>(ce_stream_),
                                      reinterpret_cast<CUdeviceptr>(v.base[d.flag_rank] + d.flag_off), d.flag_value,
                                      CU_STREAM_WRITE_VALUE_DEFAULT),
             "cuStreamWriteValue64(flag)");
    if (d.counter_value) {
        check_cu(drv.cuStreamWriteValue64(reinterpret_cast<CUstream>(ce_stream_),
                                          reinterpret_cast<CUdeviceptr>(v.base[v.rank] + d.counter_off),
                                          d.counter_value, CU_STREAM_WRITE_VALUE_DEFAULT),
                 "cuStreamWriteValue64(counter)");
    }
    copies_.fetch_add(1, std::memory_order_relaxed);
}

void Context::host_signal(const HostSignalDesc& d) {
    const HeapView& v = heap_.view();
    if (d.rank >= static_cast<uint32_t>(v.world) || d.off + 8 > v.size) {
        throw kiwi::error("kiwi::p2p: host signal out of the heap's range");
    }
    std::lock_guard<std::mutex> g(ce_mu_);
    check_cu(driver().cuStreamWriteValue64(reinterpret_cast<CUstream>(ce_stream_),
                                           reinterpret_cast<CUdeviceptr>(v.base[d.rank] + d.off), d.value,
                                           CU_STREAM_WRITE_VALUE_DEFAULT),
             "cuStreamWriteValue64(signal)");
}

void Context::spawn_proxy_threads(size_t n, std::vector<int> cpus) {
    if (cpus.empty()) cpus = topology::poller_cpus(device_, n);
    threads_->start(n, cpus);
}

void Context::join_proxy_threads() {
    threads_->stop();
    if (ce_stream_) KIWI_CUDA_CHECK(cudaStreamSynchronize(ce_stream_));
    threads_->rethrow_if_failed();
}

GContext Context::device_context() const {
    GContext g{};
    g.heap = heap_.view();
    g.invoke = ictx_->device_context();
    g.ce_put_cb = ce_put_cb_;
    g.host_signal_cb = host_signal_cb_;
    return g;
}

}  // namespace kiwi::p2p

// ---------------------------------------------------------------------------
// Host-initiated copy-engine ping-pong (the "host" mode of the reference's
// SDMA ping-pong example, examples/invoke/README.md): no kernel; the CPU
// thread of each rank issues the copy and the peer's flag write on its own
// stream and makes the stream wait (cuStreamWaitValue64) for its own flag.
// ---------------------------------------------------------------------------
#include <chrono>

#include "kiwi/p2p/p2p_ops.hpp"

namespace kiwi::p2p {

std::vector<uint64_t> host_ce_pingpong(SymmetricHeap& heap, int peer, bool initiator, uint64_t bytes, uint32_t iters,
                                       uint32_t warmup, uint64_t src_off, uint64_t dst_off, uint64_t flag_off,
                                       double timeout_s) {
    const HeapView& v = heap.view();
    if (peer < 0 || peer >= v.world || src_off + bytes > v.size || dst_off + bytes > v.size || flag_off + 8 > v.size) {
        throw kiwi::error("host_ce_pingpong: arguments outside the heap");
    }
    const Driver& drv = driver();
    cudaStream_t st;
    KIWI_CUDA_CHECK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    auto cs = reinterpret_cast<CUstream>(st);
    auto put = [&](uint64_t value) {
        if (bytes) {
            KIWI_CUDA_CHECK(cudaMemcpyAsync(v.base[peer] + dst_off, v.base[v.rank] + src_off, bytes,
                                            cudaMemcpyDeviceToDevice, st));
        }
        check_cu(drv.cuStreamWriteValue64(cs, reinterpret_cast<CUdeviceptr>(v.base[peer] + flag_off), value,
                                          CU_STREAM_WRITE_VALUE_DEFAULT),
                 "cuStreamWriteValue64");
    };
    auto wait_own = [&](uint64_t value) {
        check_cu(drv.cuStreamWaitValue64(cs, reinterpret_cast<CUdeviceptr>(v.base[v.rank] + flag_off), value,
                                         CU_STREAM_WAIT_VALUE_GEQ),
                 "cuStreamWaitValue64");
        // Bounded host wait: poll the stream instead of blocking forever.
        const auto end = std::chrono::steady_clock::now() + std::chrono::duration<double>(timeout_s);
        while (true) {
            const cudaError_t q = cudaStreamQuery(st);
            if (q == cudaSuccess) return;
            if (q != cudaErrorNotReady) KIWI_CUDA_CHECK(q);
            if (std::chrono::steady_clock::now() > end) {
                // Release the stream's wait ourselves so nothing stays queued
                // behind it, then report.
                cudaStream_t rel;
                KIWI_CUDA_CHECK(cudaStreamCreateWithFlags(&rel, cudaStreamNonBlocking));
                check_cu(drv.cuStreamWriteValue64(reinterpret_cast<CUstream>(rel),
                                                  reinterpret_cast<CUdeviceptr>(v.base[v.rank] + flag_off), value,
                                                  CU_STREAM_WRITE_VALUE_DEFAULT),
                         "cuStreamWriteValue64(release)");
                KIWI_CUDA_CHECK(cudaStreamSynchronize(rel));
                KIWI_CUDA_CHECK(cudaStreamSynchronize(st));
                cudaStreamDestroy(rel);
                cudaStreamDestroy(st);
                throw kiwi::error("host_ce_pingpong: the peer's flag did not arrive in time");
            }
        }
    };
    std::vector<uint64_t> lat;
    lat.reserve(iters);
    for (uint32_t i = 1; i <= iters + warmup; ++i) {
        const auto t0 = std::chrono::steady_clock::now();
        if (initiator) put(i);
        wait_own(i);
        if (!initiator) {
            put(i);
        } else if (i > warmup) {
            lat.push_back(static_cast<uint64_t>(
                std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count()));
        }
    }
    KIWI_CUDA_CHECK(cudaStreamSynchronize(st));
    KIWI_CUDA_CHECK(cudaStreamDestroy(st));
    return lat;
}

}  // namespace kiwi::p2p
