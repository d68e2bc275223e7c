// GPU -> CPU queue comparators with device producers: the counterpart of the
// reference's queue-baseline harness (benchmarks/queue_baselines/README.md of
// AMDResearch/kiwi: one adapter contract, shared kernels, pinned host
// consumer, per-message validation).  The reference builds third-party FIFOs
// from their upstream headers; none of those libraries is on this machine, so
// each comparator here restates a published queue PROTOCOL in code of its own:
//
//   kiwi_spsc     this repository's ring: one warp, 16-byte message from
//                 registers (push_lanes), tags in every word, no atomics.
//   kiwi_mpsc     the same ring with a device-memory line claim per message.
//   fifo_trigger  index-publishing trigger FIFO in the style of MSCCL++'s
//                 proxy FIFO: 16-byte triggers {fst, snd} in mapped host
//                 memory, a device-memory head claimed with an atomic, the
//                 consumer's tail read over PCIe only when the cached tail says
//                 the ring is full; the producer stores fst, fences at system
//                 scope and release-stores snd (non-zero = filled); the host
//                 pops a slot when snd != 0, zeroes it and publishes its tail.
//   proxy_channel byte-reservation channel in the style of NVSHMEM's proxy
//                 channel: a request is four 8-byte entries in mapped host
//                 memory, each carrying 32 payload bits and a lap-parity flag,
//                 reserved with a device-memory byte counter after a system
//                 fence; the host accepts a request when all four flags carry
//                 the lap's parity (no clearing) and publishes the bytes it
//                 consumed.
//   raw_store     the floor, not a queue: one warp-wide 64-byte store of the
//                 message and its sequence number into a host line, no
//                 capacity check (latency mode only).
//
// Modes: latency (one warp; push, host pop, host ack into a host word the
// warp polls; per-iteration %globaltimer), throughput (W warps x N messages,
// one host consumer thread, wall-clock messages per second), push_cost (SM
// cycles per push with a ring large enough never to wrap).  Every device wait
// is bounded; a timeout sets the status word and the warp stops.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstring>
#include <string>
#include <vector>

#include "kiwi/bench/gpu_bench.hpp"
#include "kiwi/bench/host_server.hpp"
#include "kiwi/ptx.cuh"
#include "kiwi/queue/queue.hpp"

namespace kiwi::bench {

namespace {

using queue::MemKind;
using queue::detail::Block;

enum QbMode : int { kModeLatency = 0, kModeThroughput = 1, kModePushCost = 2 };
enum QbQueue : int { kKiwiSpsc = 0, kKiwiMpsc = 1, kFifoTrigger = 2, kProxyChannel = 3, kRawStore = 4 };

/// Payload check word of message `seq`: both halves of a message are derived
/// from its sequence number, so a consumer can validate what it read.
KIWI_HD uint64_t qb_check(uint64_t seq) { return (seq * 0x9E3779B97F4A7C15ull) | 1ull; }

// ---------------------------------------------------------------- device sides

struct KiwiSpscDev {
    queue::SpscD2HHandle h;
    /// Warp-collective: lane 0 carries seq, lane 1 the check word.
    KIWI_DEV Status push(uint64_t seq, uint64_t check, uint64_t timeout_ns) {
        const uint64_t word = ptx::lane_id() == 0 ? seq : check;
        ptx::Deadline dl(timeout_ns);
        while (!h.push_lanes(word, 16, 0)) {
            if (dl.expired()) return Status::kTimeout;
        }
        return Status::kOk;
    }
};

struct KiwiMpscDev {
    queue::MpscD2HHandle h;
    KIWI_DEV Status push(uint64_t seq, uint64_t check, uint64_t timeout_ns) {
        const uint64_t word = ptx::lane_id() == 0 ? seq : check;
        ptx::Deadline dl(timeout_ns);
        while (!h.push_lanes(word, 16, 0)) {
            if (dl.expired()) return Status::kTimeout;
        }
        return Status::kOk;
    }
};

struct FifoTriggerDev {
    uint64_t* ring;               // [cap][2] {fst, snd} in mapped host memory
    unsigned long long* head;     // device memory
    const uint64_t* tail;         // mapped host memory, written by the consumer
    uint64_t cap;                 // power of two
    uint64_t tail_cache;          // per warp (lane 0)
    KIWI_DEV Status push(uint64_t seq, uint64_t check, uint64_t timeout_ns) {
        uint32_t st = 0;
        if (ptx::lane_id() == 0) {
            const uint64_t hd = atomicAdd(head, 1ull);
            if (hd >= tail_cache + cap) {
                ptx::Deadline dl(timeout_ns);
                while (hd >= (tail_cache = ptx::ld_volatile_u64(tail)) + cap) {
                    if (dl.expired()) {
                        st = static_cast<uint32_t>(Status::kTimeout);
                        break;
                    }
                }
            }
            if (st == 0) {
                uint64_t* slot = ring + 2 * (hd & (cap - 1));
                ptx::st_volatile_u64(slot, seq);
                __threadfence_system();
                ptx::st_release_sys_u64(slot + 1, check);
            }
        }
        return static_cast<Status>(__shfl_sync(0xffffffffu, st, 0));
    }
};

struct ProxyChannelDev {
    uint64_t* buf;                   // size bytes of 8-byte entries, mapped host memory
    unsigned long long* reserved;    // device memory byte counter
    const uint64_t* consumed;        // mapped host memory, written by the consumer
    uint64_t size;                   // bytes, power of two, multiple of 32
    uint64_t consumed_cache;         // per warp (lane 0)
    KIWI_DEV Status push(uint64_t seq, uint64_t check, uint64_t timeout_ns) {
        uint32_t st = 0;
        __threadfence_system();  // the channel orders the caller's earlier writes before the request
        if (ptx::lane_id() == 0) {
            const uint64_t pos = atomicAdd(reserved, 32ull);
            if (pos + 32 > consumed_cache + size) {
                ptx::Deadline dl(timeout_ns);
                while (pos + 32 > (consumed_cache = ptx::ld_volatile_u64(consumed)) + size) {
                    if (dl.expired()) {
                        st = static_cast<uint32_t>(Status::kTimeout);
                        break;
                    }
                }
            }
            if (st == 0) {
                const uint64_t flag = ((pos / size) & 1ull) ^ 1ull;  // the first lap writes 1 into zeroed memory
                uint64_t* e = buf + (pos & (size - 1)) / 8;
                const uint32_t part[4] = {static_cast<uint32_t>(seq), static_cast<uint32_t>(seq >> 32),
                                          static_cast<uint32_t>(check), static_cast<uint32_t>(check >> 32)};
#pragma unroll
                for (int i = 0; i < 4; ++i) ptx::st_volatile_u64(e + i, (static_cast<uint64_t>(part[i]) << 1) | flag);
            }
        }
        return static_cast<Status>(__shfl_sync(0xffffffffu, st, 0));
    }
};

struct RawStoreDev {
    uint64_t* lines;  // [cap][8] in mapped host memory
    uint64_t cap;
    KIWI_DEV Status push(uint64_t seq, uint64_t check, uint64_t) {
        // One 64-byte line from lanes 0..3, 16 bytes each; the sequence number
        // is the line's last word.
        const uint32_t lane = ptx::lane_id();
        if (lane < 4) {
            uint64_t* l = lines + 8 * (seq & (cap - 1));
            const uint64_t a = lane == 0 ? check : 0, b = lane == 3 ? seq : 0;
            ptx::st_volatile_v4(l + 2 * lane, static_cast<uint32_t>(a), static_cast<uint32_t>(a >> 32),
                                static_cast<uint32_t>(b), static_cast<uint32_t>(b >> 32));
        }
        return Status::kOk;
    }
};

/// The shared driver.  Latency: warp 0 of block 0 pushes, then polls the
/// host-written ack word until it equals the sequence number.  Throughput and
/// push cost: every warp pushes `iters` messages numbered (warp << 40) | i.
template <typename Q>
__global__ void __launch_bounds__(256) qb_kernel(Q q, int mode, uint64_t iters, uint64_t warmup, const uint64_t* ack,
                                                 uint64_t* lat_ns, uint64_t* warp_cycles, uint32_t* status,
                                                 uint64_t timeout_ns) {
    const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
    const uint32_t lane = ptx::lane_id();
    if (mode == kModeLatency) {
        if (warp != 0) return;
        for (uint64_t i = 0; i < warmup + iters; ++i) {
            const uint64_t seq = i + 1;
            const uint64_t t0 = ptx::globaltimer();
            Status st = q.push(seq, qb_check(seq), timeout_ns);
            if (st == Status::kOk) {
                uint32_t ok = 1;
                if (lane == 0) {
                    ptx::Deadline dl(timeout_ns);
                    while (ptx::ld_volatile_u64(ack) != seq) {
                        if (dl.expired()) {
                            ok = 0;
                            break;
                        }
                    }
                }
                if (!__shfl_sync(0xffffffffu, ok, 0)) st = Status::kTimeout;
            }
            if (st != Status::kOk) {
                if (lane == 0) atomicCAS(status, 0u, static_cast<uint32_t>(st));
                return;
            }
            if (lane == 0 && i >= warmup) lat_ns[i - warmup] = ptx::globaltimer() - t0;
        }
        return;
    }
    const uint64_t c0 = clock64();
    for (uint64_t i = 0; i < iters; ++i) {
        const uint64_t seq = (static_cast<uint64_t>(warp) << 40) | (i + 1);
        const Status st = q.push(seq, qb_check(seq), timeout_ns);
        if (st != Status::kOk) {
            if (lane == 0) atomicCAS(status, 0u, static_cast<uint32_t>(st));
            return;
        }
    }
    if (lane == 0) warp_cycles[warp] = clock64() - c0;
}

// ---------------------------------------------------------------- host sides

int pick_cpu(int cpu) {
    if (cpu >= 0) return cpu;
    int dev = 0;
    cudaGetDevice(&dev);
    const auto cpus = topology::poller_cpus(dev, 1);
    return cpus.empty() ? -1 : cpus[0];
}

struct DevWords {
    uint64_t* p = nullptr;
    explicit DevWords(size_t n) {
        KIWI_CUDA_CHECK(cudaMalloc(&p, std::max<size_t>(n, 1) * 8));
        KIWI_CUDA_CHECK(cudaMemset(p, 0, std::max<size_t>(n, 1) * 8));
    }
    ~DevWords() { cudaFree(p); }
    DevWords(const DevWords&) = delete;
    DevWords& operator=(const DevWords&) = delete;
};

inline uint64_t ld_acq(const uint64_t* p) { return __atomic_load_n(p, __ATOMIC_ACQUIRE); }
inline void st_rel(uint64_t* p, uint64_t v) { __atomic_store_n(p, v, __ATOMIC_RELEASE); }

/// Host consumer of one comparator: try_pop(seq, check) -> false when empty.
struct KiwiRingHost {
    queue::D2HRingBase* q;
    bool try_pop(uint64_t& seq, uint64_t& check) {
        alignas(16) uint64_t buf[queue::kMaxMessageBytes / 8];
        uint32_t meta = 0, bytes = 0;
        if (!q->try_pop(buf, &meta, &bytes)) return false;
        seq = buf[0];
        check = bytes >= 16 ? buf[1] : 0;
        return true;
    }
};

struct FifoTriggerHost {
    uint64_t* ring;
    uint64_t* tail_pub;
    uint64_t cap;
    uint64_t tail = 0;
    bool try_pop(uint64_t& seq, uint64_t& check) {
        uint64_t* slot = ring + 2 * (tail & (cap - 1));
        const uint64_t snd = ld_acq(slot + 1);
        if (snd == 0) return false;
        seq = __atomic_load_n(slot, __ATOMIC_RELAXED);
        check = snd;
        __atomic_store_n(slot, 0ull, __ATOMIC_RELAXED);
        __atomic_store_n(slot + 1, 0ull, __ATOMIC_RELAXED);
        st_rel(tail_pub, ++tail);
        return true;
    }
};

struct ProxyChannelHost {
    uint64_t* buf;
    uint64_t* consumed_pub;
    uint64_t size;
    uint64_t consumed = 0;
    bool try_pop(uint64_t& seq, uint64_t& check) {
        const uint64_t flag = ((consumed / size) & 1ull) ^ 1ull;
        const uint64_t* e = buf + (consumed & (size - 1)) / 8;
        uint64_t v[4];
        for (int i = 0; i < 4; ++i) {
            v[i] = ld_acq(e + i);
            if ((v[i] & 1ull) != flag) return false;
        }
        seq = (v[0] >> 1 & 0xffffffffull) | ((v[1] >> 1 & 0xffffffffull) << 32);
        check = (v[2] >> 1 & 0xffffffffull) | ((v[3] >> 1 & 0xffffffffull) << 32);
        consumed += 32;
        st_rel(consumed_pub, consumed);
        return true;
    }
};

struct RawStoreHost {
    uint64_t* lines;
    uint64_t cap;
    uint64_t next = 1;
    bool try_pop(uint64_t& seq, uint64_t& check) {
        uint64_t* l = lines + 8 * (next & (cap - 1));
        if (ld_acq(l + 7) != next) return false;
        seq = next++;
        check = qb_check(seq);  // the floor checks arrival only: the line's other stores may land later
        return true;
    }
};

template <typename Dev, typename Host>
GpuQueueBaselineResult run_qb(const GpuQueueBaselineOptions& o, Dev dev, Host host, uint64_t* ack_host,
                              const uint64_t* ack_dev) {
    GpuQueueBaselineResult r;
    r.queue = o.queue;
    r.mode = o.mode;
    const int mode = o.mode == "latency" ? kModeLatency : o.mode == "throughput" ? kModeThroughput : kModePushCost;
    const uint32_t warps = mode == kModeLatency ? 1u : o.warps;
    const uint64_t expected = mode == kModeLatency ? o.iters + o.warmup : static_cast<uint64_t>(warps) * o.iters;
    DevWords lat(mode == kModeLatency ? o.iters : 1), cyc(warps);
    uint32_t* status = nullptr;
    KIWI_CUDA_CHECK(cudaMalloc(&status, 4));
    KIWI_CUDA_CHECK(cudaMemset(status, 0, 4));
    cudaStream_t stream;
    KIWI_CUDA_CHECK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    const uint32_t threads = std::min<uint32_t>(256, 32 * warps);
    const uint32_t blocks = (32 * warps + threads - 1) / threads;
    uint64_t popped = 0, bad = 0, order_errors = 0;
    std::vector<uint64_t> next_per_warp(warps, 1);
    std::chrono::steady_clock::time_point t_start, t_end;
    try {
        launch_with_server(
            pick_cpu(o.cpu),
            [&] {
                t_start = std::chrono::steady_clock::now();
                qb_kernel<Dev><<<blocks, threads, 0, stream>>>(dev, mode, o.iters, o.warmup, ack_dev, lat.p, cyc.p,
                                                              status, o.timeout_ns);
                KIWI_CUDA_CHECK(cudaGetLastError());
            },
            [&](const std::atomic<bool>& launched, const std::atomic<bool>& quit) {
                if (mode == kModePushCost) return;  // nothing popped while the kernel runs
                uint64_t idle = 0;
                while (popped < expected && !quit.load(std::memory_order_relaxed)) {
                    uint64_t seq = 0, check = 0;
                    if (!host.try_pop(seq, check)) {
                        if ((++idle & 0xfffff) == 0 && stream_idle(stream, launched)) break;
                        continue;
                    }
                    idle = 0;
                    ++popped;
                    if (check != qb_check(seq)) ++bad;
                    if (mode == kModeLatency) {
                        if (seq != popped) ++order_errors;
                        st_rel(ack_host, seq);
                    } else {
                        const uint64_t w = seq >> 40;
                        if (w >= warps || (seq & ((1ull << 40) - 1)) != next_per_warp[w]) ++order_errors;
                        else ++next_per_warp[w];
                    }
                }
                t_end = std::chrono::steady_clock::now();
            });
        KIWI_CUDA_CHECK(cudaStreamSynchronize(stream));
        if (mode == kModePushCost) {
            t_end = std::chrono::steady_clock::now();
            // Drain what the kernel pushed, to validate it.
            uint64_t seq = 0, check = 0;
            while (popped < expected && host.try_pop(seq, check)) {
                ++popped;
                if (check != qb_check(seq)) ++bad;
            }
        }
        KIWI_CUDA_CHECK(cudaMemcpy(&r.status, status, 4, cudaMemcpyDeviceToHost));
        if (mode == kModeLatency) {
            r.lat_ns.resize(o.iters);
            KIWI_CUDA_CHECK(cudaMemcpy(r.lat_ns.data(), lat.p, o.iters * 8, cudaMemcpyDeviceToHost));
        }
        std::vector<uint64_t> c(warps);
        KIWI_CUDA_CHECK(cudaMemcpy(c.data(), cyc.p, warps * 8, cudaMemcpyDeviceToHost));
        uint64_t cmax = 0, csum = 0;
        for (uint64_t v : c) {
            cmax = std::max(cmax, v);
            csum += v;
        }
        r.cycles_per_push = mode == kModeLatency || o.iters == 0 ? 0.0
                                                                : static_cast<double>(csum) / warps / o.iters;
        (void)cmax;
    } catch (...) {
        cudaStreamDestroy(stream);
        cudaFree(status);
        throw;
    }
    cudaStreamDestroy(stream);
    cudaFree(status);
    r.messages = popped;
    r.bad = bad;
    r.order_errors = order_errors;
    r.seconds = std::chrono::duration<double>(t_end - t_start).count();
    r.ok = r.status == 0 && popped == expected && bad == 0 && order_errors == 0;
    return r;
}

}  // namespace

GpuQueueBaselineResult gpu_queue_baseline(const GpuQueueBaselineOptions& o) {
    static const char* const kQueues[] = {"kiwi_spsc", "kiwi_mpsc", "fifo_trigger", "proxy_channel", "raw_store"};
    int q = -1;
    for (int i = 0; i < 5; ++i) {
        if (o.queue == kQueues[i]) q = i;
    }
    if (q < 0) throw kiwi::error("gpu_queue_baseline: queue must be kiwi_spsc, kiwi_mpsc, fifo_trigger, proxy_channel "
                                 "or raw_store");
    if (o.mode != "latency" && o.mode != "throughput" && o.mode != "push_cost") {
        throw kiwi::error("gpu_queue_baseline: mode must be latency, throughput or push_cost");
    }
    if (o.iters < 1) throw kiwi::error("gpu_queue_baseline: iters must be positive");
    if (o.mode != "latency" && (o.warps < 1 || o.warps > 4096)) {
        throw kiwi::error("gpu_queue_baseline: warps must be in [1, 4096]");
    }
    if (q == kKiwiSpsc && o.mode != "latency" && o.warps != 1) {
        throw kiwi::error("gpu_queue_baseline: kiwi_spsc has one producer warp (use kiwi_mpsc for several)");
    }
    if (q == kRawStore && o.mode != "latency") {
        throw kiwi::error("gpu_queue_baseline: raw_store has no capacity check; latency mode only");
    }
    if (o.capacity < 2 || !is_pow2(o.capacity)) throw kiwi::error("gpu_queue_baseline: capacity must be a power of two");
    const uint64_t msgs = o.mode == "latency" ? 1 : static_cast<uint64_t>(o.warps) * o.iters;
    if (o.mode == "push_cost" && o.capacity < msgs) {
        throw kiwi::error("gpu_queue_baseline: push_cost needs capacity >= warps x iters (the ring must not wrap)");
    }
    Block ack(64, MemKind::kMappedPinned);
    uint64_t* ack_host = ack.as<uint64_t>();
    const uint64_t* ack_dev = ack.dev<const uint64_t>();
    switch (q) {
        case kKiwiSpsc: {
            queue::SPSCD2HQueue ring(o.capacity, MemKind::kMappedPinned);
            return run_qb(o, KiwiSpscDev{ring.device_handle()}, KiwiRingHost{&ring}, ack_host, ack_dev);
        }
        case kKiwiMpsc: {
            queue::MPSCD2HQueue ring(o.capacity, MemKind::kMappedPinned);
            return run_qb(o, KiwiMpscDev{ring.device_handle(o.timeout_ns)}, KiwiRingHost{&ring}, ack_host, ack_dev);
        }
        case kFifoTrigger: {
            Block ring(o.capacity * 16, MemKind::kMappedPinned), tail(64, MemKind::kMappedPinned);
            DevWords head(1);
            FifoTriggerDev d{ring.dev<uint64_t>(), reinterpret_cast<unsigned long long*>(head.p),
                             tail.dev<const uint64_t>(), o.capacity, 0};
            return run_qb(o, d, FifoTriggerHost{ring.as<uint64_t>(), tail.as<uint64_t>(), o.capacity}, ack_host,
                          ack_dev);
        }
        case kProxyChannel: {
            const uint64_t size = o.capacity * 32;
            Block buf(size, MemKind::kMappedPinned), consumed(64, MemKind::kMappedPinned);
            DevWords reserved(1);
            ProxyChannelDev d{buf.dev<uint64_t>(), reinterpret_cast<unsigned long long*>(reserved.p),
                              consumed.dev<const uint64_t>(), size, 0};
            return run_qb(o, d, ProxyChannelHost{buf.as<uint64_t>(), consumed.as<uint64_t>(), size}, ack_host,
                          ack_dev);
        }
        default: {
            Block lines(o.capacity * 64, MemKind::kMappedPinned);
            return run_qb(o, RawStoreDev{lines.dev<uint64_t>(), o.capacity}, RawStoreHost{lines.as<uint64_t>(),
                                                                                         o.capacity},
                          ack_host, ack_dev);
        }
    }
}

}  // namespace kiwi::bench
