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
    if (cpus.empty()) {
        cpus = topology::gpu_local_cpus(device_);
        if (cpus.size() > 1) cpus.erase(cpus.begin());  // keep core 0 for the OS
    }
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
