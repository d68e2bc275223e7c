// GPU drivers for kiwi::queue / kiwi::invoke: the round-trip benchmark, the
// raw PCIe floor, and correctness kernels for every queue kind.
//
// Counterparts in the reference (AMDResearch/kiwi):
//   invoke_rtt      benchmarks/invoke/bench_latency.hip.cpp (ping_pong_latency_handle_kernel)
//   pcie_floor      benchmarks/hardware/pcie_latency.hip.cpp:26-37 (pingpong_kernel)
//   d2h_push_test   tests/queue/test_chunk_queue.hip.cpp, test_push_lane_masked
//   h2d_*_test      tests/queue/test_host_to_device_concurrent, test_mpmc_h2d_concurrent
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>

#include "kiwi/invoke/progress.hpp"
#include <cstring>
#include <thread>

#include "kiwi/bench/gpu_bench.hpp"
#include "kiwi/bench/host_server.hpp"
#include "kiwi/bench/host_bench.hpp"
#include "kiwi/invoke/invoke.hpp"
#include "kiwi/queue/mailbox.cuh"
#include "kiwi/ptx.cuh"
#include "kiwi/topology.hpp"

namespace kiwi::bench {

using namespace kiwi::queue;
using kiwi::invoke::DeviceContext;

namespace {

KIWI_HD uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

KIWI_HD uint64_t pattern_word(uint64_t seed, uint64_t msg, uint32_t word) {
    return splitmix64(seed ^ (msg * 0x100000001B3ull) ^ (static_cast<uint64_t>(word) << 48));
}

KIWI_DEV uint64_t dev_xorshift(uint64_t& s) {
    s ^= s << 13;
    s ^= s >> 7;
    s ^= s << 17;
    return s;
}

/// Upper bound on helper warps that poll until their block's main warp sets a
/// stop flag (10 minutes: far above any benchmark run).
constexpr uint64_t kHelperGuardNs = 600ull * 1000000000ull;

template <typename T>
struct DevBuf {
    T* p = nullptr;
    explicit DevBuf(size_t n) {
        KIWI_CUDA_CHECK(cudaMalloc(&p, (n ? n : 1) * sizeof(T)));
        KIWI_CUDA_CHECK(cudaMemset(p, 0, (n ? n : 1) * sizeof(T)));
    }
    ~DevBuf() { cudaFree(p); }
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
};

struct PinnedFlag {
    volatile uint32_t* p = nullptr;
    PinnedFlag() {
        void* q = nullptr;
        KIWI_CUDA_CHECK(cudaHostAlloc(&q, 64, cudaHostAllocMapped | cudaHostAllocPortable));
        std::memset(q, 0, 64);
        p = static_cast<volatile uint32_t*>(q);
    }
    ~PinnedFlag() { cudaFreeHost(const_cast<uint32_t*>(p)); }
};

int pick_cpu(int cpu) {
    if (cpu >= 0) return cpu;
    int dev = 0;
    cudaGetDevice(&dev);
    const auto cpus = topology::poller_cpus(dev, 1);
    return cpus.empty() ? -1 : cpus[0];
}


}  // namespace

// ---------------------------------------------------------------------------
// GPU -> CPU -> GPU invoke round trip
// ---------------------------------------------------------------------------

struct RttShared {
    unsigned long long found;  // reply line + 1 of the newest message a poller saw
    uint64_t line;             // reply line the pollers should watch
    uint64_t word[4];          // payload of line (index line & 3)
    uint32_t stop;
};

template <typename Q>
__global__ void __launch_bounds__(256) invoke_rtt_kernel(
    DeviceContext<Q>* ctx, SpscH2DHandle reply, uint8_t cb, uint64_t iters, uint64_t warmup,
    uint32_t bytes, uint64_t* payload_buf, uint64_t seed, uint64_t* lat_ns, uint32_t* lat_cyc,
    uint64_t* totals, uint32_t* status, uint32_t poll_warps, uint64_t stagger_ns,
    uint64_t timeout_ns, volatile uint32_t* done, MailboxHandle mbox, uint32_t use_mailbox) {
    __shared__ RttShared sh;
    const uint32_t warp = threadIdx.x / 32;
    const uint32_t lane = ptx::lane_id();
    if (threadIdx.x == 0) {
        sh.found = 0;
        sh.line = reply.tail;
        sh.stop = 0;
    }
    __syncthreads();
    // Warps past the reply pollers in use (a block launched wider than the
    // benchmark needs, e.g. 1 x 64 threads as a wave64 block) have no role.
    if (warp > 0 && (use_mailbox || warp > poll_warps)) return;

    if (warp > 0) {
        // Helper pollers: keep one read of the watched reply line in flight each,
        // staggered so their reads reach host memory evenly spaced.
        __nanosleep(static_cast<uint32_t>(stagger_ns * (warp - 1)));
        const uint64_t mask = reply.capacity() - 1;
        // The main warp sets sh.stop on every exit path; the guard bounds the
        // loop regardless (far above any run's length).
        ptx::Deadline guard(kHelperGuardNs);
        while (true) {
            const bool quit = *reinterpret_cast<volatile uint32_t*>(&sh.stop) != 0 || guard.expired();
            if (__any_sync(ptx::kFullMask, quit)) break;  // warp-uniform: the loop body uses full-warp collectives
            const uint64_t line = *reinterpret_cast<volatile uint64_t*>(&sh.line);
            const uint32_t tag = lap_tag(line, reply.log2cap);
            uint4 v = make_uint4(0, 0, 0, 0);
            bool ok = true;
            if (lane < 2) {
                v = ptx::ld_volatile_v4(&reply.ring[(line & mask) * kChunksPerLine + lane]);
                ok = dev::chunk_ok(v, tag);
            }
            if (__all_sync(ptx::kFullMask, ok)) {
                const uint32_t lo = __shfl_sync(ptx::kFullMask, dev::chunk_lo(v), 1);
                const uint32_t hi = __shfl_sync(ptx::kFullMask, dev::chunk_hi(v), 1);
                if (lane == 0) {
                    reinterpret_cast<volatile uint64_t*>(sh.word)[line & 3] =
                        (static_cast<uint64_t>(hi) << 32) | lo;
                    __threadfence_block();
                    atomicMax(&sh.found, static_cast<unsigned long long>(line + 1));
                }
            }
        }
        return;
    }

    auto h = ctx->get_device_handle(0);
    MailboxHandle mb = mbox;  // local copy: the adaptive delay lives in registers
    uint64_t s = seed ? seed : 0x9E3779B97F4A7C15ull;
    uint32_t st = 0;
    bool ok = true;
    const uint64_t total = iters + warmup;
    uint64_t t_begin = 0, c_begin = 0;
    for (uint64_t i = 0; i < total; ++i) {
        const uint64_t x = dev_xorshift(s);
        if (i == warmup) {
            t_begin = ptx::globaltimer();
            c_begin = ptx::clock64();
        }
        if (bytes != 8) {
            if (lane == 0) payload_buf[0] = x;
            __syncwarp();
        }
        const uint64_t t0 = ptx::globaltimer();
        const uint64_t c0 = ptx::clock64();
        if (use_mailbox) {
            // The public call/return path: invoke(seq, x) + mirrored mailbox reply.
            uint64_t w = 0;
            const uint32_t seq = static_cast<uint32_t>(i + 1);
            const Status cs = bytes == 8 ? h.call(cb, mb, seq, w, timeout_ns, x)
                                         : Status::kBadArgument;
            const uint64_t t1 = ptx::globaltimer();
            const uint64_t c1 = ptx::clock64();
            if (cs != Status::kOk) {
                st = static_cast<uint32_t>(cs);
                break;
            }
            if (w != x + 1) ok = false;
            if (i >= warmup && lane == 0) {
                lat_ns[i - warmup] = t1 - t0;
                lat_cyc[i - warmup] = static_cast<uint32_t>(c1 - c0);
            }
            continue;
        }
        {
            ptx::Deadline pdl(timeout_ns);
            bool pushed = false;
            while (!(pushed = (bytes == 8 ? h.invoke(cb, x) : h.invoke_global(cb, payload_buf, bytes)))) {
                if (pdl.expired()) break;
            }
            if (!pushed) {
                st = static_cast<uint32_t>(Status::kTimeout);
                break;
            }
        }
        uint64_t w = 0;
        if (poll_warps == 0) {
            uint32_t b, m;
            if (reply.pop(w, b, m, timeout_ns) != Status::kOk) {
                st = static_cast<uint32_t>(Status::kTimeout);
                break;
            }
            w = ptx::bcast64(w, 0);
        } else {
            const uint64_t want = reply.tail + 1;
            ptx::Deadline dl(timeout_ns);
            bool timed_out = false;
            while (*reinterpret_cast<volatile unsigned long long*>(&sh.found) < want) {
                if (dl.expired()) {
                    timed_out = true;
                    break;
                }
            }
            if (timed_out) {
                st = static_cast<uint32_t>(Status::kTimeout);
                break;
            }
            w = reinterpret_cast<volatile uint64_t*>(sh.word)[reply.tail & 3];
            reply.advance(1);
            if (lane == 0) *reinterpret_cast<volatile uint64_t*>(&sh.line) = reply.tail;
        }
        const uint64_t t1 = ptx::globaltimer();
        const uint64_t c1 = ptx::clock64();
        if (w != x + 1) ok = false;
        if (i >= warmup && lane == 0) {
            lat_ns[i - warmup] = t1 - t0;
            lat_cyc[i - warmup] = static_cast<uint32_t>(c1 - c0);
        }
    }
    if (lane == 0) {
        totals[0] = ptx::globaltimer() - t_begin;
        totals[1] = ptx::clock64() - c_begin;
        status[0] = st;
        status[1] = ok ? 1u : 0u;
        *reinterpret_cast<volatile uint32_t*>(&sh.stop) = 1;
    }
    ctx->save_device_handle(0, h);
    reply.flush_consumer_index();
    __syncwarp();
    if (lane == 0) {
        __threadfence_system();
        *done = 1;
    }
}

template <typename Q>
static RttResult run_invoke_rtt(const RttConfig& cfg) {
    if (cfg.payload_bytes < 8 || cfg.payload_bytes > kMaxMessageBytes) {
        throw kiwi::error("invoke_rtt: payload_bytes must be in [8, 4096]");
    }
    if (cfg.poll_warps > 7) throw kiwi::error("invoke_rtt: poll_warps must be <= 7");
    kiwi::invoke::Context<Q> ctx(1, cfg.capacity, MemKind::kMappedPinned);
    SPSCH2DQueue reply(64, MemKind::kMappedPinned);
    ReplyMailbox mailbox(MemKind::kMappedPinned, cfg.stagger_ns, cfg.initial_delay_ns, cfg.pipeline, cfg.adaptive,
                         cfg.demote);
    uint64_t callbacks = 0;
    if (cfg.mailbox && cfg.payload_bytes != 8) throw kiwi::error("invoke_rtt: the mailbox path sends 8-byte payloads");
    const uint8_t cb = cfg.mailbox ? ctx.register_call(std::function<uint64_t(uint64_t)>([&](uint64_t v) {
                                                           ++callbacks;
                                                           return v + 1;
                                                       }),
                                                       mailbox)
                                   : ctx.register_raw_callback(
        [&](const uint8_t* p, uint32_t n) {
            uint64_t v;
            std::memcpy(&v, p, 8);
            v += 1;
            while (!reply.try_push(&v, 8, n)) host::cpu_relax();
            ++callbacks;
        },
        cfg.payload_bytes);
    if (cfg.mailbox && cfg.poll_warps) throw kiwi::error("invoke_rtt: poll_warps applies to ring replies only");

    DevBuf<uint64_t> payload(kMaxMessageBytes / 8);
    {
        std::vector<uint64_t> pat(kMaxMessageBytes / 8);
        for (size_t i = 0; i < pat.size(); ++i) pat[i] = pattern_word(cfg.seed, 0, static_cast<uint32_t>(i));
        KIWI_CUDA_CHECK(cudaMemcpy(payload.p, pat.data(), kMaxMessageBytes, cudaMemcpyHostToDevice));
    }
    DevBuf<uint64_t> lat(cfg.iters);
    DevBuf<uint32_t> cyc(cfg.iters);
    DevBuf<uint64_t> totals(2);
    DevBuf<uint32_t> status(2);
    PinnedFlag done;
    cudaStream_t stream;
    KIWI_CUDA_CHECK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));

    const int cpu = pick_cpu(cfg.cpu);
    const uint32_t used = 32 * (1 + (cfg.mailbox ? 0 : cfg.poll_warps));
    if (cfg.block_threads && (cfg.block_threads % 32 || cfg.block_threads < used || cfg.block_threads > 256)) {
        throw kiwi::error("invoke_rtt: block_threads must be a multiple of 32 in [warps used, 256]");
    }
    const uint32_t threads = cfg.block_threads ? cfg.block_threads : used;
    launch_with_server(
        cpu,
        [&] {
            invoke_rtt_kernel<Q><<<1, threads, 0, stream>>>(
                ctx.device_context(), reply.device_handle(), cb, cfg.iters, cfg.warmup, cfg.payload_bytes,
                payload.p, cfg.seed, lat.p, cyc.p, totals.p, status.p, cfg.poll_warps,
                /*stagger_ns=*/cfg.poll_warps ? 800 / cfg.poll_warps : 0, cfg.timeout_ns, done.p,
                mailbox.device_handle(), cfg.mailbox ? 1u : 0u);
            KIWI_CUDA_CHECK(cudaGetLastError());
        },
        [&](const std::atomic<bool>& launched, const std::atomic<bool>& quit) {
            auto poll = ctx.poll_state(0);
            uint64_t idle = 0;
            while (!quit.load(std::memory_order_relaxed)) {
                if (poll.ready()) {
                    ctx.progress(0);
                    poll.refresh();
                    idle = 0;
                    continue;
                }
                if (*done.p) break;
                if ((++idle & 0xfffff) == 0 && stream_idle(stream, launched)) break;
            }
            ctx.progress(0);
        });
    KIWI_CUDA_CHECK(cudaStreamSynchronize(stream));
    cudaStreamDestroy(stream);

    RttResult r;
    r.lat_ns.resize(cfg.iters);
    std::vector<uint32_t> c32(cfg.iters);
    uint64_t tot[2];
    uint32_t stv[2];
    KIWI_CUDA_CHECK(cudaMemcpy(r.lat_ns.data(), lat.p, cfg.iters * 8, cudaMemcpyDeviceToHost));
    KIWI_CUDA_CHECK(cudaMemcpy(c32.data(), cyc.p, cfg.iters * 4, cudaMemcpyDeviceToHost));
    KIWI_CUDA_CHECK(cudaMemcpy(tot, totals.p, sizeof(tot), cudaMemcpyDeviceToHost));
    KIWI_CUDA_CHECK(cudaMemcpy(stv, status.p, sizeof(stv), cudaMemcpyDeviceToHost));
    r.lat_cycles.assign(c32.begin(), c32.end());
    r.total_ns = tot[0];
    r.total_cycles = tot[1];
    r.status = stv[0];
    r.callbacks = callbacks;
    r.ok = stv[0] == 0 && stv[1] == 1 && callbacks == cfg.iters + cfg.warmup;
    ctx.check_device_errors();
    return r;
}

RttResult invoke_rtt(const RttConfig& cfg) {
    return cfg.mpsc ? run_invoke_rtt<MPSCD2HQueue>(cfg) : run_invoke_rtt<SPSCD2HQueue>(cfg);
}

// ---------------------------------------------------------------------------
// Raw PCIe store-and-poll floor
// ---------------------------------------------------------------------------

__global__ void pcie_floor_kernel(uint64_t* d2h, const uint64_t* h2d, uint64_t iters,
                                  uint64_t warmup, uint64_t* lat_ns, uint32_t* lat_cyc,
                                  uint64_t* totals, uint32_t* status, uint64_t timeout_ns) {
    if (threadIdx.x != 0) return;
    uint64_t t_begin = 0, c_begin = 0;
    for (uint64_t i = 0; i < iters + warmup; ++i) {
        if (i == warmup) {
            t_begin = ptx::globaltimer();
            c_begin = ptx::clock64();
        }
        const uint64_t t0 = ptx::globaltimer();
        const uint64_t c0 = ptx::clock64();
        ptx::st_volatile_u64(d2h, i + 1);
        ptx::Deadline dl(timeout_ns);
        while (ptx::ld_volatile_u64(h2d) != i + 1) {
            if (dl.expired()) {
                status[0] = static_cast<uint32_t>(Status::kTimeout);
                ptx::st_volatile_u64(d2h, ~0ull);
                return;
            }
        }
        const uint64_t t1 = ptx::globaltimer();
        const uint64_t c1 = ptx::clock64();
        if (i >= warmup) {
            lat_ns[i - warmup] = t1 - t0;
            lat_cyc[i - warmup] = static_cast<uint32_t>(c1 - c0);
        }
    }
    totals[0] = ptx::globaltimer() - t_begin;
    totals[1] = ptx::clock64() - c_begin;
    status[1] = 1;
    ptx::fence_sys();
    ptx::st_volatile_u64(d2h, ~0ull);
}

RttResult pcie_floor(uint64_t iters, uint64_t warmup, int cpu, uint64_t timeout_ns) {
    detail::Block words(128, MemKind::kMappedPinned);
    volatile uint64_t* d2h = words.as<volatile uint64_t>();
    volatile uint64_t* h2d = words.as<volatile uint64_t>() + 8;  // separate cache line
    DevBuf<uint64_t> lat(iters);
    DevBuf<uint32_t> cyc(iters);
    DevBuf<uint64_t> totals(2);
    DevBuf<uint32_t> status(2);
    cudaStream_t stream;
    KIWI_CUDA_CHECK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    launch_with_server(
        pick_cpu(cpu),
        [&] {
            pcie_floor_kernel<<<1, 32, 0, stream>>>(const_cast<uint64_t*>(d2h), const_cast<uint64_t*>(h2d), iters,
                                                    warmup, lat.p, cyc.p, totals.p, status.p, timeout_ns);
            KIWI_CUDA_CHECK(cudaGetLastError());
        },
        [&](const std::atomic<bool>& launched, const std::atomic<bool>& quit) {
            uint64_t expect = 1;
            uint64_t idle = 0;
            while (!quit.load(std::memory_order_relaxed)) {
                const uint64_t v = *d2h;
                if (v == ~0ull) break;
                if (v == expect) {
                    *h2d = v;
                    ++expect;
                    idle = 0;
                } else if ((++idle & 0xfffff) == 0 && stream_idle(stream, launched)) {
                    break;
                }
            }
        });
    KIWI_CUDA_CHECK(cudaStreamSynchronize(stream));
    cudaStreamDestroy(stream);
    RttResult r;
    r.lat_ns.resize(iters);
    std::vector<uint32_t> c32(iters);
    uint64_t tot[2];
    uint32_t stv[2];
    KIWI_CUDA_CHECK(cudaMemcpy(r.lat_ns.data(), lat.p, iters * 8, cudaMemcpyDeviceToHost));
    KIWI_CUDA_CHECK(cudaMemcpy(c32.data(), cyc.p, iters * 4, cudaMemcpyDeviceToHost));
    KIWI_CUDA_CHECK(cudaMemcpy(tot, totals.p, sizeof(tot), cudaMemcpyDeviceToHost));
    KIWI_CUDA_CHECK(cudaMemcpy(stv, status.p, sizeof(stv), cudaMemcpyDeviceToHost));
    r.lat_cycles.assign(c32.begin(), c32.end());
    r.total_ns = tot[0];
    r.total_cycles = tot[1];
    r.status = stv[0];
    r.ok = stv[0] == 0 && stv[1] == 1;
    return r;
}


// ---------------------------------------------------------------------------
// Grid polling of mapped host memory (reference:
// benchmarks/hardware/bench_host_mapped_grid_poll.hip.cpp): per round, block 0
// publishes the round number into a host-mapped count slot after `delay_ns`;
// lane 0 of every warp of the other blocks polls it; each of those blocks then
// stores its own ack line (host-mapped, 64 bytes apart, plain release stores:
// no host-memory atomics) and block 0 waits for every ack.  One GPU clock
// (%globaltimer) times publish -> each warp's observation and publish -> last
// ack.  Cooperative launch: every block is resident, so no poller waits on a
// publisher that is not running.  Every wait is bounded.
// ---------------------------------------------------------------------------

__global__ void grid_poll_kernel(uint64_t* count_slot, uint64_t* acks, uint32_t rounds, uint64_t delay_ns,
                                 uint64_t* pub_ns, uint64_t* obs_ns, uint64_t* ack_ns, uint32_t* status,
                                 uint64_t timeout_ns) {
    const uint32_t warps = blockDim.x / 32;
    const uint32_t warp = threadIdx.x / 32;
    const uint32_t lane = ptx::lane_id();
    __shared__ int s_fail;
    if (threadIdx.x == 0) s_fail = 0;
    __syncthreads();
    for (uint32_t r = 1; r <= rounds; ++r) {
        if (blockIdx.x == 0) {
            if (threadIdx.x == 0) {
                const uint64_t t_start = ptx::globaltimer();
                while (ptx::globaltimer() - t_start < delay_ns) {
                }
                const uint64_t t_pub = ptx::globaltimer();
                ptx::st_release_sys_u64(count_slot, r);
                pub_ns[r - 1] = t_pub;
                for (uint32_t b = 1; b < gridDim.x; ++b) {
                    ptx::Deadline dl(timeout_ns);
                    while (ptx::ld_acquire_sys_u64(acks + 8 * b) != r) {
                        if (dl.expired()) {
                            status[0] = static_cast<uint32_t>(Status::kTimeout);
                            s_fail = 1;
                            break;
                        }
                    }
                    if (s_fail) break;
                }
                ack_ns[r - 1] = ptx::globaltimer() - t_pub;
            }
        } else {
            if (lane == 0) {
                ptx::Deadline dl(timeout_ns);
                uint64_t v = ptx::ld_acquire_sys_u64(count_slot);
                while (v < r) {
                    if (dl.expired()) {
                        status[0] = static_cast<uint32_t>(Status::kTimeout);
                        s_fail = 1;
                        break;
                    }
                    v = ptx::ld_acquire_sys_u64(count_slot);
                }
                obs_ns[(static_cast<uint64_t>(r) - 1) * (gridDim.x - 1) * warps + (blockIdx.x - 1) * warps + warp] =
                    ptx::globaltimer();
            }
            __syncthreads();
            if (threadIdx.x == 0 && !s_fail) ptx::st_release_sys_u64(acks + 8 * blockIdx.x, r);
        }
        __syncthreads();
        if (*reinterpret_cast<volatile int*>(&s_fail) || *reinterpret_cast<volatile uint32_t*>(status) != 0) return;
    }
}

GridPollResult grid_poll(uint32_t blocks, uint32_t threads, uint32_t rounds, uint64_t delay_ns, uint64_t timeout_ns) {
    if (blocks < 2 || threads < 32 || threads % 32 || threads > 1024 || rounds < 1) {
        throw kiwi::error("grid_poll: blocks >= 2, threads a multiple of 32 in [32, 1024], rounds >= 1");
    }
    if (delay_ns > 1000000000ull || timeout_ns > 60000000000ull) {
        throw kiwi::error("grid_poll: delay_ns at most 1 s and timeout_ns at most 60 s");
    }
    int dev = 0, per_sm = 0, sms = 0, coop = 0;
    KIWI_CUDA_CHECK(cudaGetDevice(&dev));
    KIWI_CUDA_CHECK(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev));
    KIWI_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    KIWI_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, grid_poll_kernel, static_cast<int>(threads), 0));
    if (!coop || static_cast<int64_t>(blocks) > static_cast<int64_t>(per_sm) * sms) {
        throw kiwi::error("grid_poll: the grid must fit on the GPU at once (cooperative launch)");
    }
    detail::Block slots(64 * (blocks + 1), MemKind::kMappedPinned);  // count line, then one ack line per block
    uint64_t* count_slot = slots.as<uint64_t>();
    uint64_t* acks = slots.as<uint64_t>() + 8;
    const uint32_t pollers = (blocks - 1) * (threads / 32);
    DevBuf<uint64_t> pub(rounds), obs(static_cast<uint64_t>(rounds) * pollers), ackt(rounds);
    DevBuf<uint32_t> status(1);
    void* args[] = {&count_slot, &acks, &rounds, &delay_ns, &pub.p, &obs.p, &ackt.p, &status.p, &timeout_ns};
    KIWI_CUDA_CHECK(cudaLaunchCooperativeKernel(reinterpret_cast<void*>(grid_poll_kernel), dim3(blocks), dim3(threads),
                                                args, 0, nullptr));
    KIWI_CUDA_CHECK(cudaDeviceSynchronize());
    std::vector<uint64_t> p(rounds), o(static_cast<size_t>(rounds) * pollers), a(rounds);
    uint32_t st = 0;
    KIWI_CUDA_CHECK(cudaMemcpy(p.data(), pub.p, rounds * 8, cudaMemcpyDeviceToHost));
    KIWI_CUDA_CHECK(cudaMemcpy(o.data(), obs.p, o.size() * 8, cudaMemcpyDeviceToHost));
    KIWI_CUDA_CHECK(cudaMemcpy(a.data(), ackt.p, rounds * 8, cudaMemcpyDeviceToHost));
    KIWI_CUDA_CHECK(cudaMemcpy(&st, status.p, 4, cudaMemcpyDeviceToHost));
    GridPollResult r;
    r.blocks = blocks;
    r.pollers = pollers;
    r.status = st;
    r.ok = st == 0;
    if (!r.ok) return r;
    std::vector<double> first, last, acklat;
    for (uint32_t k = 0; k < rounds; ++k) {
        uint64_t lo = ~0ull, hi = 0;
        for (uint32_t w = 0; w < pollers; ++w) {
            const uint64_t t = o[static_cast<size_t>(k) * pollers + w];
            lo = std::min(lo, t);
            hi = std::max(hi, t);
        }
        first.push_back(static_cast<double>(lo > p[k] ? lo - p[k] : 0));
        last.push_back(static_cast<double>(hi > p[k] ? hi - p[k] : 0));
        acklat.push_back(static_cast<double>(a[k]));
    }
    auto pct = [](std::vector<double> v, double q) {
        std::sort(v.begin(), v.end());
        return v[std::min(v.size() - 1, static_cast<size_t>(q * (v.size() - 1) + 0.5))];
    };
    r.first_observe_p50_ns = pct(first, 0.5);
    r.last_observe_p50_ns = pct(last, 0.5);
    r.last_observe_p99_ns = pct(last, 0.99);
    r.ack_p50_ns = pct(acklat, 0.5);
    r.ack_p99_ns = pct(acklat, 0.99);
    return r;
}

// ---------------------------------------------------------------------------
// Round-trip protocol lab: measures store-and-poll variants so the invoke
// reply path can use the fastest one on this platform.
//   pollers   warps polling the host ack (0: the storing thread polls itself)
//   mirrors   the host writes the ack to this many separate 128-byte lines;
//             poller p reads line p % mirrors
//   stagger   ns between pollers' first reads (then free-running)
//   fence     fence.sc.sys after the GPU's store
//   pipeline  one thread keeps `pipeline` loads in flight (staggered)
// ---------------------------------------------------------------------------

struct LabShared {
    unsigned long long found;
    uint32_t stop;
};

__global__ void __launch_bounds__(288) rtt_lab_kernel(uint64_t* d2h, const uint64_t* acks, uint32_t mirrors,
                                                     uint64_t iters, uint64_t warmup, uint64_t* lat_ns,
                                                     uint32_t* lat_cyc, uint64_t* totals, uint32_t* status,
                                                     uint32_t pollers, uint32_t stagger_ns, uint32_t fence,
                                                     uint32_t pipeline, uint64_t timeout_ns, uint32_t initial_delay_ns) {
    __shared__ LabShared sh;
    const uint32_t warp = threadIdx.x / 32;
    const uint32_t lane = ptx::lane_id();
    if (threadIdx.x == 0) {
        sh.found = 0;
        sh.stop = 0;
    }
    __syncthreads();
    if (warp > 0) {
        if (lane != 0) return;
        const uint32_t p = warp - 1;
        const uint64_t* a = acks + static_cast<uint64_t>(p % mirrors) * 16;
        const uint64_t t_start = ptx::globaltimer() + static_cast<uint64_t>(stagger_ns) * p;
        while (ptx::globaltimer() < t_start) {
        }
        ptx::Deadline guard(kHelperGuardNs);  // sh.stop ends the loop; the guard bounds it regardless
        while (!*reinterpret_cast<volatile uint32_t*>(&sh.stop) && !guard.expired()) {
            const uint64_t v = ptx::ld_volatile_u64(a);
            if (v > *reinterpret_cast<volatile unsigned long long*>(&sh.found)) atomicMax(&sh.found, v);
        }
        return;
    }
    if (lane != 0) return;
    uint64_t t_begin = 0, c_begin = 0;
    for (uint64_t i = 0; i < iters + warmup; ++i) {
        if (i == warmup) {
            t_begin = ptx::globaltimer();
            c_begin = ptx::clock64();
        }
        const uint64_t want = i + 1;
        const uint64_t t0 = ptx::globaltimer();
        const uint64_t c0 = ptx::clock64();
        ptx::st_volatile_u64(d2h, want);
        if (fence) ptx::fence_sys();
        if (initial_delay_ns) {
            const uint64_t td = ptx::globaltimer();
            while (ptx::globaltimer() < td + initial_delay_ns) {
            }
        }
        ptx::Deadline dl(timeout_ns);
        bool ok = true;
        if (pollers > 0) {
            while (*reinterpret_cast<volatile unsigned long long*>(&sh.found) < want) {
                if (dl.expired()) { ok = false; break; }
            }
        } else if (pipeline <= 1) {
            while (ptx::ld_volatile_u64(acks) < want) {
                if (dl.expired()) { ok = false; break; }
            }
        } else {
            // Keep `pipeline` (<= 4) loads in flight, each issued stagger_ns apart.
            const uint64_t* a0 = acks;
            const uint64_t* a1 = acks + (1 % mirrors) * 16;
            const uint64_t* a2 = acks + (2 % mirrors) * 16;
            const uint64_t* a3 = acks + (3 % mirrors) * 16;
            uint64_t v0 = ptx::ld_volatile_u64(a0), v1 = 0, v2 = 0, v3 = 0;
            uint64_t t = ptx::globaltimer();
            while (ptx::globaltimer() < t + stagger_ns) {}
            v1 = ptx::ld_volatile_u64(a1);
            if (pipeline > 2) { t = ptx::globaltimer(); while (ptx::globaltimer() < t + stagger_ns) {} v2 = ptx::ld_volatile_u64(a2); }
            if (pipeline > 3) { t = ptx::globaltimer(); while (ptx::globaltimer() < t + stagger_ns) {} v3 = ptx::ld_volatile_u64(a3); }
            while (true) {
                if (v0 >= want) break;
                v0 = ptx::ld_volatile_u64(a0);
                if (v1 >= want) break;
                v1 = ptx::ld_volatile_u64(a1);
                if (pipeline > 2) { if (v2 >= want) break; v2 = ptx::ld_volatile_u64(a2); }
                if (pipeline > 3) { if (v3 >= want) break; v3 = ptx::ld_volatile_u64(a3); }
                if (dl.expired()) { ok = false; break; }
            }
        }
        const uint64_t t1 = ptx::globaltimer();
        const uint64_t c1 = ptx::clock64();
        if (!ok) {
            status[0] = static_cast<uint32_t>(Status::kTimeout);
            break;
        }
        if (i >= warmup) {
            lat_ns[i - warmup] = t1 - t0;
            lat_cyc[i - warmup] = static_cast<uint32_t>(c1 - c0);
        }
    }
    totals[0] = ptx::globaltimer() - t_begin;
    totals[1] = ptx::clock64() - c_begin;
    status[1] = 1;
    *reinterpret_cast<volatile uint32_t*>(&sh.stop) = 1;
    ptx::fence_sys();
    ptx::st_volatile_u64(d2h, ~0ull);
}

RttResult rtt_lab(uint64_t iters, uint64_t warmup, uint32_t pollers, uint32_t mirrors, uint32_t stagger_ns,
                  uint32_t fence, uint32_t pipeline, int cpu, uint32_t initial_delay_ns) {
    if (pollers > 8 || mirrors == 0 || mirrors > 8 || pipeline > 4) throw kiwi::error("rtt_lab: bad arguments");
    detail::Block words(64 + 8 * 128, MemKind::kMappedPinned);
    volatile uint64_t* d2h = words.as<volatile uint64_t>();
    volatile uint64_t* acks = words.as<volatile uint64_t>() + 8;  // ack mirror m at acks[16 * m]
    DevBuf<uint64_t> lat(iters);
    DevBuf<uint32_t> cyc(iters);
    DevBuf<uint64_t> totals(2);
    DevBuf<uint32_t> status(2);
    cudaStream_t stream;
    KIWI_CUDA_CHECK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    launch_with_server(
        pick_cpu(cpu),
        [&] {
            rtt_lab_kernel<<<1, 32 * (1 + pollers), 0, stream>>>(
                const_cast<uint64_t*>(d2h), const_cast<uint64_t*>(acks), mirrors, iters, warmup, lat.p, cyc.p,
                totals.p, status.p, pollers, stagger_ns, fence, pipeline, 2000000000ull, initial_delay_ns);
            KIWI_CUDA_CHECK(cudaGetLastError());
        },
        [&](const std::atomic<bool>& launched, const std::atomic<bool>& quit) {
            uint64_t expect = 1, idle = 0;
            while (!quit.load(std::memory_order_relaxed)) {
                const uint64_t v = *d2h;
                if (v == ~0ull) break;
                if (v == expect) {
                    for (uint32_t m = 0; m < mirrors; ++m) acks[16 * m] = v;
                    ++expect;
                    idle = 0;
                } else if ((++idle & 0xfffff) == 0 && stream_idle(stream, launched)) {
                    break;
                }
            }
        });
    KIWI_CUDA_CHECK(cudaStreamSynchronize(stream));
    cudaStreamDestroy(stream);
    RttResult r;
    r.lat_ns.resize(iters);
    std::vector<uint32_t> c32(iters);
    uint64_t tot[2];
    uint32_t stv[2];
    KIWI_CUDA_CHECK(cudaMemcpy(r.lat_ns.data(), lat.p, iters * 8, cudaMemcpyDeviceToHost));
    KIWI_CUDA_CHECK(cudaMemcpy(c32.data(), cyc.p, iters * 4, cudaMemcpyDeviceToHost));
    KIWI_CUDA_CHECK(cudaMemcpy(tot, totals.p, sizeof(tot), cudaMemcpyDeviceToHost));
    KIWI_CUDA_CHECK(cudaMemcpy(stv, status.p, sizeof(stv), cudaMemcpyDeviceToHost));
    r.lat_cycles.assign(c32.begin(), c32.end());
    r.total_ns = tot[0];
    r.total_cycles = tot[1];
    r.status = stv[0];
    r.ok = stv[0] == 0 && stv[1] == 1;
    return r;
}



// ---------------------------------------------------------------------------
// Platform assumptions of the wire format (reference category:
// tests/queue/test_hardware_assumptions.hip.cpp).  One 64-byte line is
// rewritten `iters` times while the other side reads it as fast as it can.
// D2H modes (the GPU writes round i, the host reads with aligned 8-byte loads;
// "v4" = one 16-byte store per chunk, "u64" = two 8-byte stores):
//   0 v4 / 1 u64: raw words {i, ~i}       3-4: raw {~i, i} (v4 / u64)
//   2 v4 / 5 u64: tagged {i:16 | i:16}    6-7: tagged {mix16(i) | i:16}
//   8 v4:         {i:16 | ~i:16}          (every word self-checking)
// torn8 counts 8-byte halves whose two words came from different rounds,
// tag_ahead those whose high word was the newer one, torn_word 32-bit words
// whose two 16-bit halves disagree (the property the wire format needs).
// H2D (atomicity_h2d_test): the host rewrites tagged words with 8-byte
// stores for a fixed time, one GPU warp reads whole chunks with 16-byte loads.
// ---------------------------------------------------------------------------

KIWI_HD uint32_t mix16(uint32_t x) {
    x &= 0xffffu;
    return ((x * 40503u) ^ (x >> 7) ^ 0x5bd1u) & 0xffffu;
}

/// The 32-bit word of round i in mode m, and whether mode m is raw.
KIWI_HD uint32_t atom_word(uint32_t mode, uint32_t i, bool high) {
    switch (mode) {
        case 0:
        case 1: return high ? ~i : i;
        case 3:
        case 4: return high ? i : ~i;
        case 2:
        case 5: return tagged_word(i, i);
        case 6:
        case 7: return tagged_word(mix16(i), i);
        default: return (i & 0xffffu) | ((~i & 0xffffu) << 16);
    }
}

KIWI_HD bool atom_v4(uint32_t mode) { return mode == 0 || mode == 2 || mode == 3 || mode == 6 || mode == 8; }

__global__ void atomicity_writer_kernel(Chunk* line, uint32_t iters, uint32_t mode, volatile uint32_t* done) {
    const uint32_t lane = ptx::lane_id();
    const bool v4 = atom_v4(mode);
    for (uint32_t i = 1; i <= iters; ++i) {
        if (lane < 4) {
            const uint32_t lo = atom_word(mode, i, false), hi = atom_word(mode, i, true);
            if (v4) {
                ptx::st_volatile_v4(&line[lane], lo, hi, lo, hi);
            } else {
                const uint64_t h = static_cast<uint64_t>(lo) | (static_cast<uint64_t>(hi) << 32);
                ptx::st_volatile_u64(&line[lane].lo, h);
                ptx::st_volatile_u64(&line[lane].hi, h);
            }
        }
        __syncwarp();
    }
    if (lane == 0) {
        ptx::fence_sys();
        *done = 1;
    }
}

namespace {

/// Round (low 16 bits for tagged modes, full for raw) carried by a word.
uint32_t word_round(uint32_t mode, uint32_t w, bool high) {
    switch (mode) {
        case 0:
        case 1: return high ? ~w : w;
        case 3:
        case 4: return high ? w : ~w;
        case 8: return w & 0xffffu;
        default: return w >> 16;
    }
}

bool word_torn(uint32_t mode, uint32_t w) {
    switch (mode) {
        case 2:
        case 5: return (w & 0xffffu) != (w >> 16);
        case 6:
        case 7: return (w & 0xffffu) != mix16(w >> 16);
        case 8: return ((w ^ (w >> 16)) & 0xffffu) != 0xffffu;
        default: return false;  // raw words carry no redundancy
    }
}

/// Classifies one 8-byte half read while the line was being rewritten.
void classify_half(uint32_t mode, uint64_t h, AtomicityResult& r) {
    const uint32_t w0 = static_cast<uint32_t>(h), w1 = static_cast<uint32_t>(h >> 32);
    const bool bad_word = word_torn(mode, w0) || word_torn(mode, w1);
    r.torn_word += word_torn(mode, w0) + word_torn(mode, w1);
    const bool raw = mode <= 1 || mode == 3 || mode == 4;
    const uint32_t r0 = word_round(mode, w0, false), r1 = word_round(mode, w1, true);
    if ((r0 != r1 || bad_word) && r.samples.size() < 64) r.samples.push_back(h);
    // The wire format's assumption: a word being rewritten reads as its old
    // value, its new value or zero.  Count reads that it does not explain.
    if (raw) {
        if (r0 != r1 && w0 != 0 && w1 != 0) ++r.torn_nonzero;
    } else {
        r.torn_nonzero += (word_torn(mode, w0) && w0 != 0) + (word_torn(mode, w1) && w1 != 0);
    }
    if (r0 == r1) return;
    ++r.torn8;
    const bool high_newer = raw ? r1 > r0 : ((r1 - r0) & 0xffffu) < 0x8000u;
    if (high_newer) ++r.tag_ahead;
}

}  // namespace

AtomicityResult atomicity_test(uint32_t iters, uint32_t mode) {
    if (mode > 8) throw kiwi::error("atomicity_test: mode 0..8");
    detail::Block mem(128, MemKind::kMappedPinned);
    PinnedFlag done;
    Chunk* line = mem.as<Chunk>();
    cudaStream_t stream;
    KIWI_CUDA_CHECK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    atomicity_writer_kernel<<<1, 32, 0, stream>>>(line, iters, mode, done.p);
    KIWI_CUDA_CHECK(cudaGetLastError());
    AtomicityResult r;
    uint64_t idle = 0;
    while (!*done.p) {
        for (int c = 0; c < 4; ++c) {
            const uint64_t a = host::load_half(&line[c].lo);
            const uint64_t b = host::load_half(&line[c].hi);
            ++r.reads;
            classify_half(mode, a, r);
            classify_half(mode, b, r);
            if (a != b) ++r.split16;
        }
        if ((++idle & 0xfffff) == 0 && cudaStreamQuery(stream) != cudaErrorNotReady) break;
    }
    KIWI_CUDA_CHECK(cudaStreamSynchronize(stream));
    cudaStreamDestroy(stream);
    const uint64_t last = host::load_half(&line[3].hi);
    r.final_ok = static_cast<uint32_t>(last) == atom_word(mode, iters, false) &&
                 static_cast<uint32_t>(last >> 32) == atom_word(mode, iters, true);
    return r;
}

// Protocol-level check, as a ring reader sees it: the GPU writes round i
// (i = 1, 2, ...) into one line and waits (bounded) for the host to
// acknowledge it before writing round i+1; the host polls for round i and, in
// every 8-byte half whose tags read as round i, checks the data.  format 0 is
// the wire format (16-bit tag in every word), format 1 a {data32, tag32} half.
// accepted_bad must stay 0; torn counts halves that were neither round.

KIWI_HD uint32_t proto_data(uint32_t i, uint32_t half) { return (i * 2654435761u) ^ (half * 0x9e3779b9u) ^ 0xa5a5a5a5u; }

KIWI_HD uint64_t proto_half(uint32_t format, uint32_t i, uint32_t half) {
    const uint32_t d = proto_data(i, half);
    return format == 0 ? pack_half(d, i) : (static_cast<uint64_t>(d) | (static_cast<uint64_t>(i) << 32));
}

__global__ void protocol_writer_kernel(Chunk* line, const volatile uint32_t* ack, uint32_t iters, uint32_t format,
                                       uint32_t* status, uint64_t timeout_ns) {
    const uint32_t lane = ptx::lane_id();
    for (uint32_t i = 1; i <= iters; ++i) {
        if (lane < 4) {
            const uint64_t a = proto_half(format, i, 2 * lane), b = proto_half(format, i, 2 * lane + 1);
            ptx::st_volatile_v4(&line[lane], static_cast<uint32_t>(a), static_cast<uint32_t>(a >> 32),
                                static_cast<uint32_t>(b), static_cast<uint32_t>(b >> 32));
        }
        __syncwarp();
        if (lane == 0) {
            ptx::Deadline dl(timeout_ns);
            while (*ack != i) {
                if (dl.expired()) {
                    status[0] = 1;
                    break;
                }
            }
        }
        if (__shfl_sync(ptx::kFullMask, lane == 0 ? status[0] : 0u, 0)) return;
    }
}

ProtocolResult atomicity_protocol_test(uint32_t iters, uint32_t format) {
    detail::Block mem(128, MemKind::kMappedPinned);
    PinnedFlag ack;
    DevBuf<uint32_t> status(2);
    Chunk* line = mem.as<Chunk>();
    cudaStream_t stream;
    KIWI_CUDA_CHECK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    protocol_writer_kernel<<<1, 32, 0, stream>>>(line, ack.p, iters, format, status.p, 2000000000ull);
    KIWI_CUDA_CHECK(cudaGetLastError());
    ProtocolResult r;
    const auto tag_of = [&](uint64_t h, uint32_t i) {
        return format == 0 ? half_has_tag(h, i) : static_cast<uint32_t>(h >> 32) == i;
    };
    const auto data_of = [&](uint64_t h) { return format == 0 ? half_data(h) : static_cast<uint32_t>(h); };
    const auto give_up = std::chrono::steady_clock::now() + std::chrono::seconds(60);
    for (uint32_t i = 1; i <= iters; ++i) {
        uint32_t seen = 0;  // halves already accepted this round (bit mask)
        uint64_t spins = 0;
        while (seen != 0xffu) {
            for (uint32_t c = 0; c < 4; ++c) {
                for (uint32_t k = 0; k < 2; ++k) {
                    const uint32_t half = 2 * c + k;
                    if (seen & (1u << half)) continue;
                    const uint64_t h = host::load_half(k ? &line[c].hi : &line[c].lo);
                    ++r.reads;
                    if (tag_of(h, i)) {
                        seen |= 1u << half;
                        if (data_of(h) != proto_data(i, half)) {
                            ++r.accepted_bad;
                            if (r.samples.size() < 32) r.samples.push_back(h);
                        }
                    } else if (h != proto_half(format, i - 1, half) && !(i == 1 && h == 0)) {
                        ++r.torn;
                    }
                }
            }
            if ((++spins & 0xffff) == 0 && std::chrono::steady_clock::now() > give_up) break;
        }
        if (seen != 0xffu) break;
        ++r.rounds;
        *ack.p = i;
    }
    KIWI_CUDA_CHECK(cudaStreamSynchronize(stream));
    uint32_t st[2];
    KIWI_CUDA_CHECK(cudaMemcpy(st, status.p, sizeof(st), cudaMemcpyDeviceToHost));
    cudaStreamDestroy(stream);
    r.ok = st[0] == 0 && r.rounds == iters;
    return r;
}

__global__ void atomicity_reader_kernel(const Chunk* line, volatile uint32_t* done, unsigned long long* counts,
                                        uint64_t max_reads, uint64_t timeout_ns) {
    const uint32_t lane = ptx::lane_id();
    uint64_t reads = 0, torn_word = 0, torn8 = 0, split16 = 0;
    ptx::Deadline dl(timeout_ns);
    bool timed_out = false;
    while (reads < max_reads) {
        if (*done) break;
        if (dl.expired()) {
            timed_out = true;
            break;
        }
        if (lane < 4) {
            const uint4 v = ptx::ld_volatile_v4(&line[lane]);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if ((w[j] & 0xffffu) != mix16(w[j] >> 16)) {
                    const unsigned long long k = atomicAdd(&counts[5], 1ull);
                    if (k < 32) counts[8 + k] = w[j];
                    if (w[j] != 0) atomicAdd(&counts[6], 1ull);
                    ++torn_word;
                }
            }
            torn8 += (v.x != v.y) + (v.z != v.w);
            split16 += v.x != v.z;
        }
        ++reads;
    }
    if (lane < 4) {
        atomicAdd(&counts[0], reads);
        atomicAdd(&counts[1], torn_word);
        atomicAdd(&counts[2], torn8);
        atomicAdd(&counts[3], split16);
        if (timed_out) atomicAdd(&counts[4], 1ull);
    }
}

AtomicityResult atomicity_h2d_test(uint32_t duration_ms) {
    detail::Block mem(128, MemKind::kMappedPinned);
    PinnedFlag done;
    Chunk* line = mem.as<Chunk>();
    DevBuf<unsigned long long> counts(40);
    cudaStream_t stream;
    KIWI_CUDA_CHECK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    const uint64_t timeout_ns = (static_cast<uint64_t>(duration_ms) + 10000) * 1000000ull;
    atomicity_reader_kernel<<<1, 32, 0, stream>>>(static_cast<const Chunk*>(device_address(line, MemKind::kMappedPinned)),
                                                  done.p, counts.p, ~0ull, timeout_ns);
    KIWI_CUDA_CHECK(cudaGetLastError());
    const auto t_end = std::chrono::steady_clock::now() + std::chrono::milliseconds(duration_ms);
    for (uint32_t i = 1;; ++i) {
        const uint64_t t = tagged_word(mix16(i), i);
        const uint64_t h = t | (t << 32);
        for (int c = 0; c < 4; ++c) {
            host::store_half(&line[c].lo, h);
            host::store_half(&line[c].hi, h);
        }
        if ((i & 1023) == 0 && std::chrono::steady_clock::now() > t_end) break;
    }
    std::atomic_thread_fence(std::memory_order_seq_cst);
    *done.p = 1;
    KIWI_CUDA_CHECK(cudaStreamSynchronize(stream));
    cudaStreamDestroy(stream);
    unsigned long long c[40];
    KIWI_CUDA_CHECK(cudaMemcpy(c, counts.p, sizeof(c), cudaMemcpyDeviceToHost));
    AtomicityResult r;
    for (unsigned long long k = 0; k < c[5] && k < 32; ++k) r.samples.push_back(c[8 + k]);
    r.reads = c[0] / 4;
    r.torn_word = c[1];
    r.torn_nonzero = c[6];
    r.torn8 = c[2];
    r.split16 = c[3];
    r.final_ok = c[4] == 0;
    return r;
}

// ---------------------------------------------------------------------------
// Invoke throughput and push cost (reference: benchmarks/invoke/
// bench_throughput.hip.cpp:39, bench_overhead.hip.cpp:54-119)
// ---------------------------------------------------------------------------

__global__ void invoke_throughput_kernel(DeviceContext<SPSCD2HQueue>* ctx, uint8_t cb, uint32_t msgs,
                                         uint32_t payload_words, uint64_t* t_begin_end, uint32_t* status,
                                         uint64_t timeout_ns) {
    auto h = ctx->get_device_handle(blockIdx.x);
    const uint32_t lane = ptx::lane_id();
    if (blockIdx.x == 0 && lane == 0) t_begin_end[0] = ptx::globaltimer();
    for (uint32_t i = 0; i < msgs; ++i) {
        const uint64_t w = (static_cast<uint64_t>(blockIdx.x) << 32) | i;
        ptx::Deadline dl(timeout_ns);
        while (!h.queue.push_lanes(w, payload_words * 8, cb)) {
            if (dl.expired()) {
                if (lane == 0) status[0] = 1;
                ctx->save_device_handle(blockIdx.x, h);
                return;
            }
        }
    }
    ctx->save_device_handle(blockIdx.x, h);
    __syncwarp();
    if (lane == 0) atomicMax(reinterpret_cast<unsigned long long*>(&t_begin_end[1]), ptx::globaltimer());
}

ThroughputResult invoke_throughput(uint32_t endpoints, uint32_t threads, uint32_t msgs_per_endpoint,
                                   uint32_t payload_bytes, uint64_t capacity) {
    if (payload_bytes % 8 || payload_bytes > 256) throw kiwi::error("invoke_throughput: payload 8..256, multiple of 8");
    kiwi::invoke::Context<SPSCD2HQueue> ctx(endpoints, capacity, MemKind::kMappedPinned);
    std::atomic<uint64_t> count{0};
    const uint8_t cb = ctx.register_raw_callback(
        [&](const uint8_t*, uint32_t) { count.fetch_add(1, std::memory_order_relaxed); },
        kiwi::invoke::CallbackBase::kAnySize);
    DevBuf<uint64_t> t(2);
    DevBuf<uint32_t> status(1);
    kiwi::invoke::ProgressThreads<SPSCD2HQueue> pt(ctx);
    int dev = 0;
    cudaGetDevice(&dev);
    pt.start(threads, topology::poller_cpus(dev, threads));
    invoke_throughput_kernel<<<endpoints, 32>>>(ctx.device_context(), cb, msgs_per_endpoint, payload_bytes / 8, t.p,
                                                status.p, 2000000000ull);
    KIWI_CUDA_CHECK(cudaGetLastError());
    KIWI_CUDA_CHECK(cudaDeviceSynchronize());
    const uint64_t want = static_cast<uint64_t>(endpoints) * msgs_per_endpoint;
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(10);
    while (count.load() < want && std::chrono::steady_clock::now() < deadline) std::this_thread::yield();
    pt.stop();
    uint64_t tv[2];
    uint32_t st = 0;
    KIWI_CUDA_CHECK(cudaMemcpy(tv, t.p, sizeof(tv), cudaMemcpyDeviceToHost));
    KIWI_CUDA_CHECK(cudaMemcpy(&st, status.p, 4, cudaMemcpyDeviceToHost));
    ThroughputResult r;
    r.messages = count.load();
    r.device_ns = tv[1] - tv[0];
    r.ok = st == 0 && r.messages == want;
    return r;
}

__global__ void push_cost_kernel(SpscD2HHandle h, uint32_t msgs, uint32_t bytes, uint64_t* cycles, uint32_t* status) {
    const uint32_t lane = ptx::lane_id();
    uint64_t total = 0;
    for (uint32_t i = 0; i < msgs; ++i) {
        const uint64_t c0 = ptx::clock64();
        bool ok = h.push_lanes(i, bytes, 0);
        const uint64_t c1 = ptx::clock64();
        if (!ok) {
            // Ring full: wait for the host without counting the wait.
            ptx::Deadline dl(2000000000ull);
            while (!h.push_lanes(i, bytes, 0)) {
                if (dl.expired()) {
                    if (lane == 0) status[0] = 1;
                    return;
                }
            }
        } else {
            total += c1 - c0;
        }
    }
    if (lane == 0) cycles[0] = total;
}

PushCostResult push_cost(uint32_t msgs, uint32_t bytes) {
    SPSCD2HQueue q(1 << 16, MemKind::kMappedPinned);
    DevBuf<uint64_t> cyc(1);
    DevBuf<uint32_t> status(1);
    cudaStream_t stream;
    KIWI_CUDA_CHECK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    push_cost_kernel<<<1, 32, 0, stream>>>(q.device_handle(), msgs, bytes, cyc.p, status.p);
    KIWI_CUDA_CHECK(cudaGetLastError());
    alignas(64) uint8_t buf[kMaxMessageBytes];
    uint32_t meta, b;
    uint64_t popped = 0, idle = 0;
    while (popped < msgs) {
        if (q.try_pop(buf, &meta, &b)) {
            ++popped;
        } else if ((++idle & 0xfffff) == 0 && cudaStreamQuery(stream) != cudaErrorNotReady) {
            break;
        }
    }
    KIWI_CUDA_CHECK(cudaStreamSynchronize(stream));
    cudaStreamDestroy(stream);
    uint64_t c = 0;
    uint32_t st = 0;
    KIWI_CUDA_CHECK(cudaMemcpy(&c, cyc.p, 8, cudaMemcpyDeviceToHost));
    KIWI_CUDA_CHECK(cudaMemcpy(&st, status.p, 4, cudaMemcpyDeviceToHost));
    PushCostResult r;
    r.cycles_per_push = msgs ? static_cast<double>(c) / msgs : 0;
    r.ok = st == 0 && popped == msgs;
    return r;
}

/// SM cycles one warp spends per invoke (reference: bench_overhead.hip.cpp:54-119):
/// mode 0 = invoke(cb, int32, float, uint64), a 16-byte argument image
/// serialised in registers; mode 1 = invoke_lane_masked with the even lanes
/// active (16 messages per call).  Calls that find the ring full are retried
/// without counting the wait.
__global__ void invoke_cost_kernel(DeviceContext<SPSCD2HQueue>* ctx, uint8_t cb, uint32_t calls, int mode,
                                   uint64_t* cycles, uint32_t* status) {
    auto h = ctx->get_device_handle(0);
    const uint32_t lane = ptx::lane_id();
    uint64_t total = 0;
    for (uint32_t i = 0; i < calls; ++i) {
        const int32_t a = static_cast<int32_t>(i);
        const float b = 0.5f * static_cast<float>(i);
        // invoke takes warp-uniform arguments; the lane-masked form sends each lane's own
        const uint64_t c = mode == 0 ? i : ((static_cast<uint64_t>(lane) << 32) | i);
        auto once = [&]() { return mode == 0 ? h.invoke(cb, a, b, c) : h.invoke_lane_masked(cb, (lane & 1) == 0, a, b, c); };
        const uint64_t c0 = ptx::clock64();
        const bool ok = once();
        const uint64_t c1 = ptx::clock64();
        if (ok) {
            total += c1 - c0;
            continue;
        }
        ptx::Deadline dl(2000000000ull);
        while (!once()) {
            if (dl.expired()) {
                if (lane == 0) status[0] = 1;
                ctx->save_device_handle(0, h);
                return;
            }
        }
    }
    ctx->save_device_handle(0, h);
    if (lane == 0) cycles[0] = total;
}

InvokeCostResult invoke_cost(uint32_t calls, bool lane_masked) {
    kiwi::invoke::Context<SPSCD2HQueue> ctx(1, 1 << 16, MemKind::kMappedPinned);
    std::atomic<uint64_t> count{0};
    const uint8_t cb = ctx.register_raw_callback(
        [&](const uint8_t*, uint32_t n) {
            if (n == 16) count.fetch_add(1, std::memory_order_relaxed);
        },
        kiwi::invoke::CallbackBase::kAnySize);
    DevBuf<uint64_t> cyc(1);
    DevBuf<uint32_t> status(1);
    cudaStream_t stream;
    KIWI_CUDA_CHECK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    invoke_cost_kernel<<<1, 32, 0, stream>>>(ctx.device_context(), cb, calls, lane_masked ? 1 : 0, cyc.p, status.p);
    KIWI_CUDA_CHECK(cudaGetLastError());
    const uint64_t want = static_cast<uint64_t>(calls) * (lane_masked ? 16 : 1);
    uint64_t idle = 0;
    while (count.load() < want) {
        if (ctx.progress(0) == 0 && (++idle & 0xfffff) == 0 && cudaStreamQuery(stream) != cudaErrorNotReady) {
            ctx.progress(0);
            break;
        }
    }
    KIWI_CUDA_CHECK(cudaStreamSynchronize(stream));
    cudaStreamDestroy(stream);
    uint64_t c = 0;
    uint32_t st = 0;
    KIWI_CUDA_CHECK(cudaMemcpy(&c, cyc.p, 8, cudaMemcpyDeviceToHost));
    KIWI_CUDA_CHECK(cudaMemcpy(&st, status.p, 4, cudaMemcpyDeviceToHost));
    InvokeCostResult r;
    r.cycles_per_call = calls ? static_cast<double>(c) / calls : 0;
    r.messages = count.load();
    r.ok = st == 0 && r.messages == want;
    return r;
}

// ---------------------------------------------------------------------------
// Device-to-host push correctness
// ---------------------------------------------------------------------------

enum PushMode : int { kModeGlobal = 0, kModeLanes = 1, kModeReg = 2, kModeLaneMasked = 3 };

struct LaneMsg {
    uint64_t w[8];
};

template <uint32_t S>
struct RegMsg {
    uint8_t b[S];
};

/// Fills a register message byte pattern with fully unrolled stores so the
/// object stays in registers (a runtime-indexed loop would put it in local memory).
template <uint32_t S>
KIWI_DEV void fill_reg_msg(RegMsg<S>& m, uint64_t seed, uint64_t id) {
#pragma unroll
    for (uint32_t w = 0; w < (S + 7) / 8; ++w) {
        const uint64_t v = pattern_word(seed, id, w);
#pragma unroll
        for (uint32_t k = 0; k < 8; ++k) {
            if (w * 8 + k < S) m.b[w * 8 + k] = static_cast<uint8_t>(v >> (8 * k));
        }
    }
}

KIWI_DEV void fill_words(uint64_t* dst, uint64_t seed, uint64_t msg, uint32_t nwords) {
    for (uint32_t k = ptx::lane_id(); k < nwords; k += 32) dst[k] = pattern_word(seed, msg, k);
}

/// Message id of warp w, sequence s: unique across warps.
KIWI_HD uint64_t msg_id(uint32_t w, uint64_t s) { return (static_cast<uint64_t>(w) << 32) | s; }

/// Retries a push until it succeeds or `timeout_ns` passes (then records kTimeout).
template <typename H, typename F>
KIWI_DEV bool push_bounded(H& h, F&& push, uint64_t timeout_ns = 2000000000ull) {
    ptx::Deadline dl(timeout_ns);
    while (!push()) {
        if (dl.expired()) {
            dev::report(h.err, Status::kTimeout, site_d2h_push, 0);
            return false;
        }
    }
    return true;
}

template <typename H, int MODE, uint32_t REG_BYTES>
__global__ void __launch_bounds__(128) d2h_push_kernel(H* handles, uint32_t msgs, const uint32_t* sizes,
                                                       uint32_t nsizes, uint64_t seed,
                                                       uint64_t seq_base, uint64_t* scratch) {
    const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
    const uint32_t lane = ptx::lane_id();
    H h = handles[std::is_same<H, SpscD2HHandle>::value ? 0 : 0];
    uint64_t* buf = scratch + static_cast<uint64_t>(warp) * (kMaxMessageBytes / 8 + 1);
    for (uint32_t i = 0; i < msgs; ++i) {
        const uint64_t seq = seq_base + i;
        const uint64_t id = msg_id(warp, seq);
        const uint32_t meta = (warp << 20) | static_cast<uint32_t>(seq & 0xfffff);
        if constexpr (MODE == kModeGlobal) {
            const uint32_t bytes = sizes[seq % nsizes];
            fill_words(buf, seed, id, (bytes + 7) / 8);
            __syncwarp();
            if (!push_bounded(h, [&] { return h.push_global(buf, bytes, meta); })) return;
            __syncwarp();
        } else if constexpr (MODE == kModeLanes) {
            const uint32_t bytes = sizes[seq % nsizes];
            const uint64_t w = pattern_word(seed, id, lane);
            if (!push_bounded(h, [&] { return h.push_lanes(w, bytes, meta); })) return;
        } else if constexpr (MODE == kModeReg) {
            RegMsg<REG_BYTES> m;
            fill_reg_msg(m, seed, id);
            if (!push_bounded(h, [&] { return h.push_reg(m, meta); })) return;
        } else {
            // Each lane pushes its own message; lane-specific id and size.
            const uint64_t lid = msg_id(warp, seq * 32 + lane);
            const bool active = ((seq * 7 + lane * 3) % 5) != 0;
            const uint32_t bytes = static_cast<uint32_t>(8 + (seq * 13 + lane * 11) % 57);
            LaneMsg m;
#pragma unroll
            for (uint32_t k = 0; k < 8; ++k) m.w[k] = pattern_word(seed, lid, k);
            const uint32_t lmeta = (warp << 20) | static_cast<uint32_t>((seq * 32 + lane) & 0xfffff);
            if (!push_bounded(h, [&] { return h.push_lane_masked(m, bytes, lmeta, active); })) return;
        }
    }
    if constexpr (std::is_same<H, SpscD2HHandle>::value) {
        if (lane == 0 && warp == 0) handles[0] = h;
    }
}

template <typename H, int MODE, uint32_t REG_BYTES>
static void launch_push(H* d_handle, uint32_t warps, uint32_t msgs, const uint32_t* d_sizes,
                        uint32_t nsizes, uint64_t seed, uint64_t seq_base, uint64_t* scratch,
                        cudaStream_t stream) {
    const uint32_t threads = warps >= 4 ? 128 : 32 * warps;
    const uint32_t blocks = (warps * 32 + threads - 1) / threads;
    d2h_push_kernel<H, MODE, REG_BYTES><<<blocks, threads, 0, stream>>>(d_handle, msgs, d_sizes, nsizes,
                                                                        seed, seq_base, scratch);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

template <typename H>
static void launch_mode(int mode, uint32_t reg_bytes, H* d_handle, uint32_t warps, uint32_t msgs,
                        const uint32_t* d_sizes, uint32_t nsizes, uint64_t seed, uint64_t seq_base,
                        uint64_t* scratch, cudaStream_t stream) {
    switch (mode) {
        case kModeGlobal:
            launch_push<H, kModeGlobal, 8>(d_handle, warps, msgs, d_sizes, nsizes, seed, seq_base, scratch, stream);
            break;
        case kModeLanes:
            launch_push<H, kModeLanes, 8>(d_handle, warps, msgs, d_sizes, nsizes, seed, seq_base, scratch, stream);
            break;
        case kModeLaneMasked:
            launch_push<H, kModeLaneMasked, 8>(d_handle, warps, msgs, d_sizes, nsizes, seed, seq_base, scratch, stream);
            break;
        case kModeReg:
            switch (reg_bytes) {
                case 8: launch_push<H, kModeReg, 8>(d_handle, warps, msgs, d_sizes, nsizes, seed, seq_base, scratch, stream); break;
                case 20: launch_push<H, kModeReg, 20>(d_handle, warps, msgs, d_sizes, nsizes, seed, seq_base, scratch, stream); break;
                case 56: launch_push<H, kModeReg, 56>(d_handle, warps, msgs, d_sizes, nsizes, seed, seq_base, scratch, stream); break;
                case 200: launch_push<H, kModeReg, 200>(d_handle, warps, msgs, d_sizes, nsizes, seed, seq_base, scratch, stream); break;
                case 512: launch_push<H, kModeReg, 512>(d_handle, warps, msgs, d_sizes, nsizes, seed, seq_base, scratch, stream); break;
                default: throw kiwi::error("d2h_push_test: reg mode sizes are 8, 20, 56, 200, 512");
            }
            break;
        default: throw kiwi::error("d2h_push_test: unknown mode");
    }
}

static bool check_payload(const uint8_t* got, uint32_t bytes, uint64_t seed, uint64_t id) {
    for (uint32_t k = 0; k < bytes; ++k) {
        const uint8_t want = static_cast<uint8_t>(pattern_word(seed, id, k / 8) >> (8 * (k % 8)));
        if (got[k] != want) return false;
    }
    return true;
}

PushTestResult d2h_push_test(const std::string& mode_name, bool mpsc, uint64_t capacity,
                             uint32_t warps, uint32_t msgs_per_warp,
                             const std::vector<uint32_t>& sizes_in, uint32_t launches,
                             uint64_t seed) {
    int mode = kModeGlobal;
    if (mode_name == "global") mode = kModeGlobal;
    else if (mode_name == "lanes") mode = kModeLanes;
    else if (mode_name == "reg") mode = kModeReg;
    else if (mode_name == "lane_masked") mode = kModeLaneMasked;
    else throw kiwi::error("d2h_push_test: mode must be global, lanes, reg or lane_masked");
    if (!mpsc && warps != 1) throw kiwi::error("d2h_push_test: SPSC takes exactly one producer warp");
    std::vector<uint32_t> sizes = sizes_in.empty() ? std::vector<uint32_t>{8} : sizes_in;
    const uint32_t reg_bytes = sizes[0];
    if (mode == kModeReg) sizes = {reg_bytes};

    std::unique_ptr<SPSCD2HQueue> sq;
    std::unique_ptr<MPSCD2HQueue> mq;
    D2HRingBase* base = nullptr;
    if (mpsc) {
        mq = std::make_unique<MPSCD2HQueue>(capacity, MemKind::kMappedPinned);
        base = mq.get();
    } else {
        sq = std::make_unique<SPSCD2HQueue>(capacity, MemKind::kMappedPinned);
        base = sq.get();
    }
    DevBuf<uint32_t> d_sizes(sizes.size());
    KIWI_CUDA_CHECK(cudaMemcpy(d_sizes.p, sizes.data(), sizes.size() * 4, cudaMemcpyHostToDevice));
    DevBuf<uint64_t> scratch(static_cast<size_t>(warps) * (kMaxMessageBytes / 8 + 1));
    DevBuf<uint8_t> d_handle(sizeof(MpscD2HHandle) > sizeof(SpscD2HHandle) ? sizeof(MpscD2HHandle)
                                                                            : sizeof(SpscD2HHandle));
    if (mpsc) {
        auto h = mq->device_handle();
        KIWI_CUDA_CHECK(cudaMemcpy(d_handle.p, &h, sizeof(h), cudaMemcpyHostToDevice));
    } else {
        auto h = sq->device_handle();
        KIWI_CUDA_CHECK(cudaMemcpy(d_handle.p, &h, sizeof(h), cudaMemcpyHostToDevice));
    }
    cudaStream_t stream;
    KIWI_CUDA_CHECK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));

    PushTestResult res;
    std::vector<uint64_t> next(warps, 0);
    alignas(64) uint8_t buf[kMaxMessageBytes];
    auto note = [&](const std::string& s) {
        if (res.first_error.empty()) res.first_error = s;
    };
    for (uint32_t l = 0; l < launches; ++l) {
        const uint64_t seq_base = static_cast<uint64_t>(l) * msgs_per_warp;
        if (mpsc) {
            launch_mode<MpscD2HHandle>(mode, reg_bytes, reinterpret_cast<MpscD2HHandle*>(d_handle.p), warps,
                                       msgs_per_warp, d_sizes.p, static_cast<uint32_t>(sizes.size()), seed,
                                       seq_base, scratch.p, stream);
        } else {
            launch_mode<SpscD2HHandle>(mode, reg_bytes, reinterpret_cast<SpscD2HHandle*>(d_handle.p), warps,
                                       msgs_per_warp, d_sizes.p, static_cast<uint32_t>(sizes.size()), seed,
                                       seq_base, scratch.p, stream);
        }
        // Expected messages this launch.
        uint64_t expected = 0;
        std::vector<std::vector<uint64_t>> plan(warps);  // lane-masked: per-warp list of (seq*32+lane)
        if (mode == kModeLaneMasked) {
            for (uint32_t w = 0; w < warps; ++w) {
                for (uint64_t s = seq_base; s < seq_base + msgs_per_warp; ++s) {
                    for (uint32_t ln = 0; ln < 32; ++ln) {
                        if (((s * 7 + ln * 3) % 5) != 0) plan[w].push_back(s * 32 + ln);
                    }
                }
                expected += plan[w].size();
            }
            std::fill(next.begin(), next.end(), 0);
        } else {
            expected = static_cast<uint64_t>(warps) * msgs_per_warp;
        }
        uint64_t got = 0;
        uint64_t idle = 0;
        while (got < expected) {
            uint32_t meta = 0, bytes = 0;
            if (!base->try_pop(buf, &meta, &bytes)) {
                if ((++idle & 0xffff) == 0) {
                    const cudaError_t q = cudaStreamQuery(stream);
                    if (q != cudaErrorNotReady) {
                        // Kernel finished; drain what is left then stop.
                        while (base->try_pop(buf, &meta, &bytes)) {
                            ++got;
                        }
                        if (got < expected) note("kernel finished with messages missing");
                        break;
                    }
                }
                continue;
            }
            ++got;
            const uint32_t w = meta >> 20;
            if (w >= warps) {
                ++res.mismatches;
                note("bad warp id in metadata");
                continue;
            }
            if (mode == kModeLaneMasked) {
                if (next[w] >= plan[w].size()) {
                    ++res.order_errors;
                    continue;
                }
                const uint64_t lseq = plan[w][next[w]++];
                if ((meta & 0xfffff) != (lseq & 0xfffff)) {
                    ++res.order_errors;
                    note("lane-masked order");
                    continue;
                }
                const uint64_t s = lseq / 32;
                const uint32_t ln = static_cast<uint32_t>(lseq % 32);
                const uint32_t want_bytes = static_cast<uint32_t>(8 + (s * 13 + ln * 11) % 57);
                if (bytes != want_bytes || !check_payload(buf, bytes, seed, msg_id(w, lseq))) {
                    ++res.mismatches;
                    note("lane-masked payload");
                }
            } else {
                const uint64_t s = seq_base + next[w];
                if ((meta & 0xfffff) != (s & 0xfffff)) {
                    ++res.order_errors;
                    note("order: warp " + std::to_string(w));
                }
                ++next[w];
                const uint32_t want_bytes = sizes[s % sizes.size()];
                if (bytes != want_bytes || !check_payload(buf, bytes, seed, msg_id(w, s))) {
                    ++res.mismatches;
                    note("payload: warp " + std::to_string(w) + " seq " + std::to_string(s) +
                         " bytes " + std::to_string(bytes));
                }
            }
        }
        res.popped += got;
        KIWI_CUDA_CHECK(cudaStreamSynchronize(stream));
        if (mode != kModeLaneMasked) std::fill(next.begin(), next.end(), 0);
    }
    cudaStreamDestroy(stream);
    res.device_error = base->error().code;
    return res;
}

// ---------------------------------------------------------------------------
// Host-to-device SPSC
// ---------------------------------------------------------------------------

__global__ void h2d_spsc_kernel(SpscH2DHandle h, uint32_t count, bool registers, uint64_t* out,
                                uint32_t* lens, uint32_t* metas, uint32_t* status, uint64_t timeout_ns) {
    const uint32_t lane = ptx::lane_id();
    for (uint32_t i = 0; i < count; ++i) {
        uint64_t* dst = out + static_cast<uint64_t>(i) * (kMaxMessageBytes / 8);
        uint32_t bytes = 0, meta = 0;
        ptx::Deadline dl(timeout_ns);
        if (registers) {
            uint64_t w;
            while (!h.try_pop(w, bytes, meta)) {
                if (dl.expired()) {
                    status[0] = static_cast<uint32_t>(Status::kTimeout);
                    h.flush_consumer_index();
                    return;
                }
            }
            if (lane < (bytes + 7) / 8) dst[lane] = w;
        } else {
            while (!h.try_pop_to(dst, bytes, meta)) {
                if (dl.expired()) {
                    status[0] = static_cast<uint32_t>(Status::kTimeout);
                    h.flush_consumer_index();
                    return;
                }
            }
        }
        if (lane == 0) {
            lens[i] = bytes;
            metas[i] = meta;
        }
    }
    h.flush_consumer_index();
}

PushTestResult h2d_spsc_test(uint64_t capacity, uint32_t count, const std::vector<uint32_t>& sizes_in,
                             bool registers, uint32_t notify_interval, uint64_t seed) {
    std::vector<uint32_t> sizes = sizes_in.empty() ? std::vector<uint32_t>{8} : sizes_in;
    for (uint32_t s : sizes) {
        if (registers && s > 248) throw kiwi::error("h2d_spsc_test: register pops hold <= 248 bytes");
    }
    SPSCH2DQueue q(capacity, MemKind::kMappedPinned, notify_interval);
    DevBuf<uint64_t> out(static_cast<size_t>(count) * (kMaxMessageBytes / 8));
    DevBuf<uint32_t> lens(count), metas(count), status(1);
    cudaStream_t stream;
    KIWI_CUDA_CHECK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    h2d_spsc_kernel<<<1, 32, 0, stream>>>(q.device_handle(), count, registers, out.p, lens.p, metas.p,
                                          status.p, 2000000000ull);
    KIWI_CUDA_CHECK(cudaGetLastError());
    std::vector<uint8_t> msg(kMaxMessageBytes);
    uint64_t spins = 0;
    bool gave_up = false;
    for (uint32_t i = 0; i < count && !gave_up; ++i) {
        const uint32_t bytes = sizes[i % sizes.size()];
        for (uint32_t k = 0; k < bytes; ++k) msg[k] = static_cast<uint8_t>(pattern_word(seed, i, k / 8) >> (8 * (k % 8)));
        while (!q.try_push(msg.data(), bytes, i)) {
            host::cpu_relax();
            if ((++spins & 0xfffff) == 0 && cudaStreamQuery(stream) != cudaErrorNotReady) {
                gave_up = true;
                break;
            }
        }
    }
    KIWI_CUDA_CHECK(cudaStreamSynchronize(stream));
    cudaStreamDestroy(stream);
    PushTestResult res;
    std::vector<uint64_t> h_out(static_cast<size_t>(count) * (kMaxMessageBytes / 8));
    std::vector<uint32_t> h_lens(count), h_metas(count);
    uint32_t st = 0;
    KIWI_CUDA_CHECK(cudaMemcpy(h_out.data(), out.p, h_out.size() * 8, cudaMemcpyDeviceToHost));
    KIWI_CUDA_CHECK(cudaMemcpy(h_lens.data(), lens.p, count * 4, cudaMemcpyDeviceToHost));
    KIWI_CUDA_CHECK(cudaMemcpy(h_metas.data(), metas.p, count * 4, cudaMemcpyDeviceToHost));
    KIWI_CUDA_CHECK(cudaMemcpy(&st, status.p, 4, cudaMemcpyDeviceToHost));
    res.device_error = st;
    for (uint32_t i = 0; i < count; ++i) {
        const uint32_t bytes = sizes[i % sizes.size()];
        const uint8_t* got = reinterpret_cast<const uint8_t*>(&h_out[static_cast<size_t>(i) * (kMaxMessageBytes / 8)]);
        if (h_lens[i] != bytes || h_metas[i] != i || !check_payload(got, bytes, seed, i)) {
            ++res.mismatches;
            if (res.first_error.empty()) res.first_error = "message " + std::to_string(i);
        } else {
            ++res.popped;
        }
    }
    if (q.consumer_position() != q.producer_position()) {
        if (res.first_error.empty()) res.first_error = "consumer position not flushed";
        ++res.mismatches;
    }
    return res;
}

// ---------------------------------------------------------------------------
// Host-to-device MPMC
// ---------------------------------------------------------------------------

__global__ void h2d_mpmc_kernel(MpmcH2DHandle h, uint64_t total, unsigned long long* consumed,
                                unsigned long long* out_count, uint64_t* out_words, uint32_t* out_meta,
                                uint32_t* out_len, uint32_t* status, uint64_t timeout_ns) {
    const uint32_t lane = ptx::lane_id();
    ptx::Deadline dl(timeout_ns);
    while (true) {
        uint64_t done = 0;
        if (lane == 0) done = ptx::ld_volatile_u64(consumed);
        done = ptx::bcast64(done);
        if (done >= total) return;
        uint64_t w;
        uint32_t bytes, meta;
        if (h.try_pop(w, bytes, meta)) {
            unsigned long long idx = 0;
            if (lane == 0) idx = atomicAdd(out_count, 1ull);
            idx = ptx::bcast64(idx);
            if (idx < total) {
                if (lane < 7) out_words[idx * 7 + lane] = w;
                if (lane == 0) {
                    out_meta[idx] = meta;
                    out_len[idx] = bytes;
                    atomicAdd(consumed, 1ull);
                }
            }
            dl = ptx::Deadline(timeout_ns);
        } else if (dl.expired()) {
            if (lane == 0) status[0] = static_cast<uint32_t>(Status::kTimeout);
            return;
        }
    }
}

PushTestResult h2d_mpmc_test(uint64_t slots, uint32_t slot_lines, uint32_t producers,
                             uint32_t msgs_per_producer, uint32_t warps, uint64_t seed) {
    MPMCH2DQueue q(slots, slot_lines, MemKind::kMappedPinned);
    const uint32_t payload = q.slot_payload_bytes() < 56 ? q.slot_payload_bytes() : 56;
    const uint64_t total = static_cast<uint64_t>(producers) * msgs_per_producer;
    DevBuf<unsigned long long> consumed(1), out_count(1);
    DevBuf<uint64_t> out_words(total * 7);
    DevBuf<uint32_t> out_meta(total), out_len(total), status(1);
    cudaStream_t stream;
    KIWI_CUDA_CHECK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    const uint32_t threads = warps >= 4 ? 128 : 32 * warps;
    const uint32_t blocks = (warps * 32 + threads - 1) / threads;
    h2d_mpmc_kernel<<<blocks, threads, 0, stream>>>(q.device_handle(), total, consumed.p, out_count.p,
                                                    out_words.p, out_meta.p, out_len.p, status.p,
                                                    2000000000ull);
    KIWI_CUDA_CHECK(cudaGetLastError());
    std::atomic<bool> stop{false};
    std::vector<std::thread> th;
    for (uint32_t p = 0; p < producers; ++p) {
        th.emplace_back([&, p] {
            uint8_t msg[64];
            for (uint32_t i = 0; i < msgs_per_producer && !stop; ++i) {
                const uint64_t id = (static_cast<uint64_t>(p) << 32) | i;
                for (uint32_t k = 0; k < payload; ++k) msg[k] = static_cast<uint8_t>(pattern_word(seed, id, k / 8) >> (8 * (k % 8)));
                while (!q.try_push(msg, payload, (p << 20) | i)) {
                    if (stop) return;
                    host::cpu_relax();
                }
            }
        });
    }
    // Watchdog: if the kernel ends early (timeout), release the producers.
    while (cudaStreamQuery(stream) == cudaErrorNotReady) std::this_thread::sleep_for(std::chrono::microseconds(50));
    stop = true;
    for (auto& t : th) t.join();
    KIWI_CUDA_CHECK(cudaStreamSynchronize(stream));
    cudaStreamDestroy(stream);
    PushTestResult res;
    std::vector<uint64_t> words(total * 7);
    std::vector<uint32_t> meta(total), len(total);
    uint32_t st = 0;
    unsigned long long cnt = 0;
    KIWI_CUDA_CHECK(cudaMemcpy(words.data(), out_words.p, words.size() * 8, cudaMemcpyDeviceToHost));
    KIWI_CUDA_CHECK(cudaMemcpy(meta.data(), out_meta.p, total * 4, cudaMemcpyDeviceToHost));
    KIWI_CUDA_CHECK(cudaMemcpy(len.data(), out_len.p, total * 4, cudaMemcpyDeviceToHost));
    KIWI_CUDA_CHECK(cudaMemcpy(&st, status.p, 4, cudaMemcpyDeviceToHost));
    KIWI_CUDA_CHECK(cudaMemcpy(&cnt, out_count.p, 8, cudaMemcpyDeviceToHost));
    res.device_error = st;
    std::vector<uint8_t> seen(total, 0);
    for (uint64_t i = 0; i < cnt && i < total; ++i) {
        const uint32_t p = meta[i] >> 20, s = meta[i] & 0xfffff;
        if (p >= producers || s >= msgs_per_producer) {
            ++res.mismatches;
            continue;
        }
        const uint64_t flat = static_cast<uint64_t>(p) * msgs_per_producer + s;
        if (seen[flat]++) ++res.order_errors;  // duplicate
        const uint64_t id = (static_cast<uint64_t>(p) << 32) | s;
        if (len[i] != payload || !check_payload(reinterpret_cast<const uint8_t*>(&words[i * 7]), payload, seed, id)) {
            ++res.mismatches;
        }
        ++res.popped;
    }
    if (res.popped != total && res.first_error.empty()) res.first_error = "missing messages";
    return res;
}

__global__ void h2d_timeout_kernel(SpscH2DHandle h, uint64_t timeout_ns, uint32_t* status) {
    uint64_t w;
    uint32_t b, m;
    const Status s = h.pop(w, b, m, timeout_ns);
    if (ptx::lane_id() == 0) status[0] = static_cast<uint32_t>(s);
}

uint32_t h2d_timeout_test(uint64_t timeout_ns) {
    SPSCH2DQueue q(16, MemKind::kMappedPinned);
    DevBuf<uint32_t> status(1);
    h2d_timeout_kernel<<<1, 32>>>(q.device_handle(), timeout_ns, status.p);
    KIWI_CUDA_CHECK(cudaGetLastError());
    KIWI_CUDA_CHECK(cudaDeviceSynchronize());
    uint32_t st = 0;
    KIWI_CUDA_CHECK(cudaMemcpy(&st, status.p, 4, cudaMemcpyDeviceToHost));
    const ErrorRecord e = q.error();
    if (st == static_cast<uint32_t>(Status::kTimeout) && e.code != st) return 0xffffffffu;  // not recorded
    return st;
}

std::vector<KernelAttr> queue_kernel_attributes() {
    std::vector<KernelAttr> out;
    auto add = [&](const char* name, const void* fn) {
        cudaFuncAttributes a{};
        KIWI_CUDA_CHECK(cudaFuncGetAttributes(&a, fn));
        out.push_back({name, static_cast<int>(a.localSizeBytes), a.numRegs});
    };
    add("invoke_rtt<SPSC>", reinterpret_cast<const void*>(&invoke_rtt_kernel<SPSCD2HQueue>));
    add("invoke_rtt<MPSC>", reinterpret_cast<const void*>(&invoke_rtt_kernel<MPSCD2HQueue>));
    add("push_global<SPSC>", reinterpret_cast<const void*>(&d2h_push_kernel<SpscD2HHandle, kModeGlobal, 8>));
    add("push_lanes<SPSC>", reinterpret_cast<const void*>(&d2h_push_kernel<SpscD2HHandle, kModeLanes, 8>));
    add("push_reg56<SPSC>", reinterpret_cast<const void*>(&d2h_push_kernel<SpscD2HHandle, kModeReg, 56>));
    add("push_reg200<SPSC>", reinterpret_cast<const void*>(&d2h_push_kernel<SpscD2HHandle, kModeReg, 200>));
    add("push_global<MPSC>", reinterpret_cast<const void*>(&d2h_push_kernel<MpscD2HHandle, kModeGlobal, 8>));
    add("push_lanes<MPSC>", reinterpret_cast<const void*>(&d2h_push_kernel<MpscD2HHandle, kModeLanes, 8>));
    add("h2d_spsc_pop", reinterpret_cast<const void*>(&h2d_spsc_kernel));
    add("h2d_mpmc_pop", reinterpret_cast<const void*>(&h2d_mpmc_kernel));
    return out;
}

}  // namespace kiwi::bench
