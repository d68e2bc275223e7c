// kiwi::invoke host API: a Context owns N endpoints (one device-to-host queue
// each) and one callback registry shared by all endpoints.
//
// Parity with the reference's Context<Q> (include/kiwi/invoke/invoke.hpp:20-139
// and internal/endpoint.hip.hpp:15-53 of AMDResearch/kiwi):
//   Context(num_endpoints, capacity), register_callback(std::function),
//   progress(endpoint, max), num_endpoints(), device_context(), raw_queue().
// B200 additions: register_raw_callback (byte-level callbacks, used by the
// Python frontend), poll_state(ep), check_device_errors(), and a host-only
// mode (no CUDA device: queues in plain host memory, device_context() null).
#pragma once

#include <cuda_runtime.h>

#include <memory>
#include <vector>

#include "kiwi/invoke/device_context.cuh"
#include "kiwi/invoke/registry.hpp"
#include "kiwi/queue/queue.hpp"

namespace kiwi::invoke {

/// One queue plus the loop that pops messages and runs their callbacks.
template <typename Queue>
class Endpoint {
public:
    Endpoint(uint64_t capacity, queue::MemKind kind, CallbackRegistry& registry)
        : queue_(std::make_unique<Queue>(capacity, kind)), registry_(registry) {}

    /// Runs up to `max_callbacks` callbacks (all visible ones if negative).
    size_t progress(int max_callbacks = -1) {
        size_t n = 0;
        uint32_t meta = 0, bytes = 0;
        while (max_callbacks < 0 || n < static_cast<size_t>(max_callbacks)) {
            if (!queue_->try_pop(buf_, &meta, &bytes)) break;
            registry_.get(meta & 0xffu).call(reinterpret_cast<const uint8_t*>(buf_), bytes);
            ++n;
        }
        return n;
    }

    Queue* queue() const { return queue_.get(); }

private:
    std::unique_ptr<Queue> queue_;
    CallbackRegistry& registry_;
    alignas(64) uint64_t buf_[queue::kMaxMessageBytes / 8];
};

template <typename Queue = queue::SPSCD2HQueue>
class Context {
public:
    using DeviceContextT = DeviceContext<Queue>;
    using DeviceHandle = typename DeviceContextT::DeviceHandle;

    Context(size_t num_endpoints, uint64_t queue_capacity,
            queue::MemKind kind = queue::default_host_kind())
        : kind_(kind), capacity_(queue_capacity) {
        if (num_endpoints == 0) throw invoke_error("kiwi::invoke: num_endpoints must be > 0");
        queue::check_capacity(queue_capacity);
        endpoints_.reserve(num_endpoints);
        for (size_t i = 0; i < num_endpoints; ++i) {
            endpoints_.push_back(std::make_unique<Endpoint<Queue>>(queue_capacity, kind, *registry_));
        }
        upload_handles();
    }

    ~Context() {
        if (d_handles_) cudaFree(d_handles_);
        if (d_context_) cudaFree(d_context_);
    }
    Context(const Context&) = delete;
    Context& operator=(const Context&) = delete;

    /// Registers a typed callback; the id is global across endpoints.  Throws
    /// if the endpoint rings cannot hold the argument message.
    template <typename... Args>
    uint8_t register_callback(std::function<void(Args...)> fn) {
        check_fits(ArgPack<Args...>::total_bytes);
        return registry_->add(std::make_unique<TypedCallback<Args...>>(std::move(fn)));
    }

    /// Registers a callback with a return value for DeviceHandle::call(): the
    /// message carries (seq, args...); the result is posted to `mailbox` under
    /// `seq`.  The mailbox must outlive the context's use of the callback.
    template <typename... Args>
    uint8_t register_call(std::function<uint64_t(Args...)> fn, queue::ReplyMailbox& mailbox) {
        queue::ReplyMailbox* mb = &mailbox;
        std::function<void(uint32_t, Args...)> thunk = [fn = std::move(fn), mb](uint32_t seq, Args... args) {
            mb->post(seq, fn(args...));
        };
        return register_callback<uint32_t, Args...>(std::move(thunk));
    }

    /// Registers a byte-level callback.  `expected_bytes` = exact payload size,
    /// or CallbackBase::kAnySize to accept any size up to kMaxMessageBytes.
    uint8_t register_raw_callback(RawCallback::Fn fn, uint32_t expected_bytes) {
        check_fits(expected_bytes == CallbackBase::kAnySize ? 0 : expected_bytes);
        return registry_->add(std::make_unique<RawCallback>(std::move(fn), expected_bytes));
    }

    size_t progress(size_t endpoint_id, int max_callbacks = -1) {
        return endpoint(endpoint_id).progress(max_callbacks);
    }

    /// Progress on every endpoint once; returns callbacks run.
    size_t progress_all(int max_per_endpoint = -1) {
        size_t n = 0;
        for (auto& ep : endpoints_) n += ep->progress(max_per_endpoint);
        return n;
    }

    size_t num_endpoints() const { return endpoints_.size(); }
    size_t num_callbacks() const { return registry_->size(); }
    uint64_t capacity() const { return capacity_; }

    /// Device pointer to the DeviceContext (null in host-only mode).
    DeviceContextT* device_context() const { return d_context_; }

    Queue* raw_queue(size_t endpoint_id) const { return endpoint(endpoint_id).queue(); }

    queue::HostPollState poll_state(size_t endpoint_id) const {
        return endpoint(endpoint_id).queue()->host_poll_state();
    }

    /// Handles as a host array (host-only mode, or to inspect the layout).
    std::vector<DeviceHandle> host_handles() const {
        std::vector<DeviceHandle> h;
        h.reserve(endpoints_.size());
        for (auto& ep : endpoints_) h.push_back(DeviceHandle{ep->queue()->device_handle()});
        return h;
    }

    /// Re-uploads fresh device handles (every queue must be drained).
    void upload_handles() {
        if (kind_ != queue::MemKind::kMappedPinned) return;
        const auto h = host_handles();
        if (!d_handles_) {
            KIWI_CUDA_CHECK(cudaMalloc(&d_handles_, h.size() * sizeof(DeviceHandle)));
            KIWI_CUDA_CHECK(cudaMalloc(&d_context_, sizeof(DeviceContextT)));
        }
        KIWI_CUDA_CHECK(cudaMemcpy(d_handles_, h.data(), h.size() * sizeof(DeviceHandle),
                                   cudaMemcpyHostToDevice));
        DeviceContextT ctx(d_handles_, static_cast<uint32_t>(h.size()));
        KIWI_CUDA_CHECK(cudaMemcpy(d_context_, &ctx, sizeof(ctx), cudaMemcpyHostToDevice));
    }

    /// Throws if device code recorded an error on any endpoint.
    void check_device_errors() const {
        for (size_t i = 0; i < endpoints_.size(); ++i) {
            const ErrorRecord e = endpoints_[i]->queue()->error();
            if (e.code != 0) {
                throw invoke_error("kiwi::invoke: endpoint " + std::to_string(i) + " device error " +
                                   status_name(static_cast<Status>(e.code)) + " at site " +
                                   std::to_string(e.site) + " (block " + std::to_string(e.rank) +
                                   ", info " + std::to_string(e.info) + ")");
            }
        }
    }

    queue::MemKind memory_kind() const { return kind_; }

private:
    Endpoint<Queue>& endpoint(size_t id) const {
        if (id >= endpoints_.size()) {
            throw std::out_of_range("kiwi::invoke: endpoint " + std::to_string(id) + " of " +
                                    std::to_string(endpoints_.size()));
        }
        return *endpoints_[id];
    }

    void check_fits(uint32_t bytes) const {
        if (bytes > queue::kMaxMessageBytes) {
            throw invoke_error("kiwi::invoke: callback arguments of " + std::to_string(bytes) +
                               " bytes exceed kMaxMessageBytes");
        }
        const uint32_t lines = queue::message_lines(bytes);
        if (lines > capacity_) {
            throw invoke_error("kiwi::invoke: callback arguments of " + std::to_string(bytes) +
                               " bytes need " + std::to_string(lines) +
                               " queue lines, but the queue capacity is " +
                               std::to_string(capacity_) + " lines");
        }
    }

    queue::MemKind kind_;
    uint64_t capacity_;
    std::unique_ptr<CallbackRegistry> registry_ = std::make_unique<CallbackRegistry>();
    std::vector<std::unique_ptr<Endpoint<Queue>>> endpoints_;
    DeviceHandle* d_handles_ = nullptr;
    DeviceContextT* d_context_ = nullptr;
};

}  // namespace kiwi::invoke
