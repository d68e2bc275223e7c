// Device side of kiwi::invoke: a kernel calls host callbacks through these.
//
// Parity with the reference's DeviceContext / DeviceHandle
// (include/kiwi/invoke/device_context.hip.hpp:19-137 of AMDResearch/kiwi):
//   invoke(cb)                      header-only message
//   invoke(cb, args...)             arguments serialised in registers (push_reg)
//   invoke_shared(cb, smem, bytes)  arguments already in shared memory
//   invoke_global(cb, ptr, bytes)   arguments in global memory (B200 addition, up to 4 KB)
//   invoke_lane_masked(cb, active, args...)  one message per active lane
// Every call is warp-collective (32 lanes on B200) and returns the push's
// result: false means the ring was full (SPSC) and nothing was sent.
//
// get_device_handle() returns a by-value copy whose SPSC producer position
// lives in registers: keep one copy per warp for the whole kernel and write it
// back with save_device_handle() before the kernel ends, or the next launch
// rewrites lines this one pushed.
#pragma once

#include "kiwi/invoke/serializer.hpp"
#include "kiwi/queue/handles.cuh"
#include "kiwi/queue/mailbox.cuh"

namespace kiwi::invoke {

template <typename QueueHandle>
struct InvokeHandle {
    QueueHandle queue;

#if defined(__CUDACC__)
    KIWI_DEV bool invoke(uint8_t callback_id) { return queue.push_lanes(0, 0, callback_id); }

    template <typename... Args>
    KIWI_DEV bool invoke(uint8_t callback_id, const Args&... args) {
        using P = ArgPack<Args...>;
        static_assert(P::total_bytes <= 512, "register-resident invoke arguments are limited to 512 bytes");
        PackedWords<P::kWords> p;
        P::pack_words(p.w, args...);
        return queue.push_reg_n(p, P::total_bytes, callback_id);
    }

    /// Call with a return value: sends (seq, args...) to a callback registered
    /// with Context::register_call and waits (bounded) for its 8-byte result in
    /// `mailbox`.  `seq` must be non-zero and differ from the previous call's on
    /// this mailbox (a per-warp counter).  Returns kTimeout if the push or the
    /// reply does not complete within `timeout_ns`.
    template <typename... Args>
    KIWI_DEV Status call(uint8_t callback_id, const queue::MailboxHandle& mailbox, uint32_t seq, uint64_t& result,
                         uint64_t timeout_ns, const Args&... args) {
        ptx::Deadline dl(timeout_ns);
        while (!invoke(callback_id, seq, args...)) {
            if (dl.expired()) return Status::kTimeout;
        }
        return mailbox.wait(seq, result, timeout_ns);
    }

    KIWI_DEV bool invoke_shared(uint8_t callback_id, const void* smem_args, uint32_t bytes) {
        return queue.push_shared(smem_args, bytes, callback_id);
    }

    KIWI_DEV bool invoke_global(uint8_t callback_id, const void* args, uint32_t bytes) {
        return queue.push_global(args, bytes, callback_id);
    }

    template <typename... Args>
    KIWI_DEV bool invoke_lane_masked(uint8_t callback_id, bool active, const Args&... args) {
        constexpr uint32_t n = ArgPack<Args...>::total_bytes;
        if constexpr (n == 0) {
            return queue.push_lane_masked(uint64_t{0}, 0, callback_id, active);
        } else {
            PackedWords<ArgPack<Args...>::kWords> p;
            ArgPack<Args...>::pack_words(p.w, args...);
            return queue.push_lane_masked(p, n, callback_id, active);
        }
    }
#endif
};

template <typename Queue>
class DeviceContext {
public:
    using DeviceHandle = InvokeHandle<typename Queue::DeviceHandle>;

    KIWI_HD DeviceContext(DeviceHandle* handles, uint32_t num_endpoints)
        : handles_(handles), num_endpoints_(num_endpoints) {}

    KIWI_HD uint32_t num_endpoints() const { return num_endpoints_; }

#if defined(__CUDACC__)
    /// Endpoint blockIdx.x (one endpoint per block).
    KIWI_DEV DeviceHandle get_device_handle() const { return get_device_handle(blockIdx.x); }

    /// Endpoint `ep`; an out-of-range id wraps modulo num_endpoints().
    KIWI_DEV DeviceHandle get_device_handle(uint32_t ep) const {
        return handles_[ep % num_endpoints_];
    }

    /// Lane 0 writes the handle back so the next launch continues from it.
    KIWI_DEV void save_device_handle(uint32_t ep, const DeviceHandle& h) const {
        if (ptx::lane_id() == 0) handles_[ep % num_endpoints_] = h;
    }
#endif

private:
    DeviceHandle* handles_;
    uint32_t num_endpoints_;
};

}  // namespace kiwi::invoke
