// Device handle of a kiwi::p2p::Context (see context.hpp).
//
// Parity with the reference's ghandle_t (apps/p2p/context.hip.hpp:54-128 of
// AMDResearch/kiwi): a move-only RAII handle over one control endpoint whose
// destructor writes the queue position back; post_desc / try_invoke for
// custom callbacks; post_put becomes post_ce_put (copy engine through the
// proxy) next to the direct NVLink put/get/signal of device.cuh.  Warp-collective.
#pragma once

#include "kiwi/invoke/device_context.cuh"
#include "kiwi/p2p/context.hpp"
#include "kiwi/p2p/device.cuh"

namespace kiwi::p2p {

#if defined(__CUDACC__)

class GHandle {
public:
    KIWI_DEV GHandle(const GContext& ctx, uint32_t endpoint)
        : ctx_(ctx), ep_(endpoint), h_(ctx.invoke->get_device_handle(endpoint)), armed_(true) {}
    KIWI_DEV ~GHandle() {
        if (armed_) ctx_.invoke->save_device_handle(ep_, h_);
    }
    KIWI_DEV GHandle(GHandle&& o) : ctx_(o.ctx_), ep_(o.ep_), h_(o.h_), armed_(o.armed_) { o.armed_ = false; }
    GHandle(const GHandle&) = delete;
    GHandle& operator=(const GHandle&) = delete;

    template <typename Desc>
    KIWI_DEV bool try_invoke(uint8_t cb, const Desc& d) {
        return h_.invoke(cb, d);
    }

    /// Posts a descriptor, retrying while the control ring is full (bounded).
    template <typename Desc>
    KIWI_DEV Status post_desc(uint8_t cb, const Desc& d, uint64_t timeout_ns = queue::kDefaultTimeoutNs) {
        ptx::Deadline dl(timeout_ns);
        while (!h_.invoke(cb, d)) {
            if (dl.expired()) return Status::kTimeout;
        }
        return Status::kOk;
    }

    /// Copy-engine put through a proxy thread (see CePutDesc).
    KIWI_DEV Status post_ce_put(const CePutDesc& d, uint64_t timeout_ns = queue::kDefaultTimeoutNs) {
        return post_desc(ctx_.ce_put_cb, d, timeout_ns);
    }

    /// Host-executed flag store into any rank's heap.
    KIWI_DEV Status post_host_signal(uint32_t rank, uint64_t off, uint64_t value,
                                     uint64_t timeout_ns = queue::kDefaultTimeoutNs) {
        HostSignalDesc d{rank, 0, off, value};
        return post_desc(ctx_.host_signal_cb, d, timeout_ns);
    }

    // Direct NVLink data path (warp-cooperative).
    KIWI_DEV void put(int rank, uint64_t dst_off, const void* src, uint64_t bytes) {
        put_warp(ctx_.heap, rank, dst_off, src, bytes);
    }
    KIWI_DEV void get(int rank, uint64_t src_off, void* dst, uint64_t bytes) {
        get_warp(ctx_.heap, rank, src_off, dst, bytes);
    }
    /// Put then signal (release), one warp.
    KIWI_DEV void put_signal(int rank, uint64_t dst_off, const void* src, uint64_t bytes, uint64_t flag_off,
                             uint64_t value, SignalOp op) {
        put_warp(ctx_.heap, rank, dst_off, src, bytes);
        __syncwarp();
        if (ptx::lane_id() == 0) signal(ctx_.heap, rank, flag_off, value, op);
    }
    KIWI_DEV Status wait_local(uint64_t flag_off, Cmp c, uint64_t want, uint64_t timeout_ns) {
        uint32_t st = 0;
        if (ptx::lane_id() == 0) {
            st = static_cast<uint32_t>(
                wait(reinterpret_cast<const uint64_t*>(ctx_.heap.base[ctx_.heap.rank] + flag_off), c, want, timeout_ns));
        }
        return static_cast<Status>(__shfl_sync(ptx::kFullMask, st, 0));
    }

    KIWI_DEV const GContext& context() const { return ctx_; }

private:
    GContext ctx_;
    uint32_t ep_;
    invoke::InvokeHandle<queue::SpscD2HHandle> h_;
    bool armed_;
};

#endif  // __CUDACC__

}  // namespace kiwi::p2p
