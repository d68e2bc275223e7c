// Host-only ring benchmark: two CPU threads ping-pong seeded uint64 payloads
// through two SPSC rings in shared host memory (the wire format and consumer
// of the GPU queues, with a CPU thread standing in for the producer warp).
//
// Counterpart of the reference's queue latency benchmark
// (benchmarks/queue/bench_latency.hip.cpp of AMDResearch/kiwi) run without a
// GPU: it measures the queue logic's own cost and the cache-line transfer
// between two cores, the floor under every GPU round trip.
#include "kiwi/bench/host_bench.hpp"

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstring>
#include <thread>

#include "kiwi/queue/queue.hpp"
#include "kiwi/topology.hpp"

namespace kiwi::bench {

namespace {
inline uint64_t now_ns() {
    return static_cast<uint64_t>(std::chrono::duration_cast<std::chrono::nanoseconds>(
                                     std::chrono::steady_clock::now().time_since_epoch())
                                     .count());
}
}  // namespace

uint64_t xorshift64(uint64_t& s) {
    // Marsaglia xorshift64 (13, 7, 17); state must be non-zero.
    s ^= s << 13;
    s ^= s >> 7;
    s ^= s << 17;
    return s;
}

HostRingResult host_ring_pingpong(uint64_t iters, uint64_t warmup, uint64_t capacity,
                                  uint32_t payload_bytes, uint64_t seed, int cpu_a, int cpu_b) {
    using namespace kiwi::queue;
    if (payload_bytes < 8 || payload_bytes > kMaxMessageBytes) {
        throw kiwi::error("host_ring_pingpong: payload_bytes must be in [8, 4096]");
    }
    SPSCD2HQueue a2b(capacity, MemKind::kHost);
    SPSCD2HQueue b2a(capacity, MemKind::kHost);
    RingWriter wa = a2b.host_writer();
    RingWriter wb = b2a.host_writer();
    const uint64_t total = iters + warmup;

    HostRingResult res;
    res.latencies_ns.resize(iters);
    std::atomic<bool> b_failed{false};
    uint64_t b_checksum = 0;

    std::thread tb([&] {
        if (cpu_b >= 0) topology::bind_current_thread({cpu_b});
        alignas(64) uint8_t buf[kMaxMessageBytes];
        uint64_t expect_seq = 0;
        uint32_t meta = 0, bytes = 0;
        for (uint64_t i = 0; i < total; ++i) {
            while (!a2b.try_pop(buf, &meta, &bytes)) host::cpu_relax();
            uint64_t v;
            std::memcpy(&v, buf, 8);
            if (meta != static_cast<uint32_t>(expect_seq) || bytes != payload_bytes) b_failed = true;
            ++expect_seq;
            b_checksum += v;
            const uint64_t reply = v + 1;
            while (!wb.try_push(&reply, 8, meta)) host::cpu_relax();
        }
    });

    if (cpu_a >= 0) topology::bind_current_thread({cpu_a});
    alignas(64) uint8_t msg[kMaxMessageBytes] = {0};
    alignas(64) uint8_t buf[kMaxMessageBytes];
    uint64_t state = seed ? seed : 0x9E3779B97F4A7C15ull;
    uint64_t checksum = 0;
    bool ok = true;
    const uint64_t t_start = now_ns();
    for (uint64_t i = 0; i < total; ++i) {
        const uint64_t v = xorshift64(state);
        std::memcpy(msg, &v, 8);
        checksum += v;
        const uint64_t t0 = now_ns();
        while (!wa.try_push(msg, payload_bytes, static_cast<uint32_t>(i))) host::cpu_relax();
        uint32_t meta = 0, bytes = 0;
        while (!b2a.try_pop(buf, &meta, &bytes)) host::cpu_relax();
        const uint64_t t1 = now_ns();
        uint64_t r;
        std::memcpy(&r, buf, 8);
        if (r != v + 1 || meta != static_cast<uint32_t>(i) || bytes != 8) ok = false;
        if (i >= warmup) res.latencies_ns[i - warmup] = t1 - t0;
    }
    const uint64_t t_end = now_ns();
    tb.join();
    res.ok = ok && !b_failed && b_checksum == checksum;
    res.checksum = checksum;
    res.total_ns = t_end - t_start;
    return res;
}

HostRingResult host_ring_stream(uint64_t messages, uint64_t capacity, uint32_t payload_bytes,
                                uint64_t seed, int cpu_a, int cpu_b) {
    using namespace kiwi::queue;
    if (payload_bytes < 8 || payload_bytes > kMaxMessageBytes) {
        throw kiwi::error("host_ring_stream: payload_bytes must be in [8, 4096]");
    }
    SPSCD2HQueue q(capacity, MemKind::kHost);
    RingWriter w = q.host_writer();
    HostRingResult res;
    uint64_t consumer_sum = 0;
    bool order_ok = true;
    std::thread tb([&] {
        if (cpu_b >= 0) topology::bind_current_thread({cpu_b});
        alignas(64) uint8_t buf[kMaxMessageBytes];
        uint32_t meta = 0, bytes = 0;
        for (uint64_t i = 0; i < messages; ++i) {
            while (!q.try_pop(buf, &meta, &bytes)) host::cpu_relax();
            uint64_t v;
            std::memcpy(&v, buf, 8);
            consumer_sum += v;
            if (meta != static_cast<uint32_t>(i)) order_ok = false;
        }
    });
    if (cpu_a >= 0) topology::bind_current_thread({cpu_a});
    alignas(64) uint8_t msg[kMaxMessageBytes] = {0};
    uint64_t state = seed ? seed : 0x9E3779B97F4A7C15ull;
    uint64_t sum = 0;
    const uint64_t t0 = now_ns();
    for (uint64_t i = 0; i < messages; ++i) {
        const uint64_t v = xorshift64(state);
        std::memcpy(msg, &v, 8);
        sum += v;
        while (!w.try_push(msg, payload_bytes, static_cast<uint32_t>(i))) host::cpu_relax();
    }
    tb.join();
    res.total_ns = now_ns() - t0;
    res.checksum = sum;
    res.ok = order_ok && consumer_sum == sum;
    return res;
}

}  // namespace kiwi::bench
