// Host-only queue benchmarks (no GPU needed).
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace kiwi::bench {

struct HostRingResult {
    std::vector<uint64_t> latencies_ns;  // per round trip (ping-pong only)
    uint64_t total_ns = 0;
    uint64_t checksum = 0;
    bool ok = false;                     // order and checksum verified
};

/// Marsaglia xorshift64 step (13, 7, 17).
uint64_t xorshift64(uint64_t& state);

/// Thread A pushes a seeded payload, thread B pops it and replies with
/// payload + 1 on a second ring; A records each round trip.
HostRingResult host_ring_pingpong(uint64_t iters, uint64_t warmup, uint64_t capacity,
                                  uint32_t payload_bytes, uint64_t seed, int cpu_a, int cpu_b);

/// Thread A streams `messages` seeded payloads; B pops and checks order and sum.
HostRingResult host_ring_stream(uint64_t messages, uint64_t capacity, uint32_t payload_bytes,
                                uint64_t seed, int cpu_a, int cpu_b);

/// One queue design measured by queue_baselines().
struct BaselineResult {
    std::string name;
    double p50_ns = 0;           // ping-pong round trip
    double p99_ns = 0;
    double msgs_per_s = 0;       // one-way streaming
    double idle_poll_ns = 0;     // one poll of an empty queue (0: not run)
    double loaded_p50_ns = 0;    // ping-pong while another pair streams (0: not run)
    double loaded_p99_ns = 0;
    double loaded_bg_msgs_per_s = 0;  // the background stream's rate meanwhile
    bool ok = false;             // order and checksums verified in every run
};

struct BaselineOptions {
    uint64_t iters = 10000, warmup = 1000, messages = 200000;
    uint32_t payload_bytes = 8;
    uint64_t capacity = 1024;
    int cpu_a = -1, cpu_b = -1;  // ping-pong / stream threads (-1: unpinned)
    uint64_t idle_polls = 0;     // 0: skip the idle-poll mode
    bool loaded = false;         // run the loaded-latency mode
    int cpu_c = -1, cpu_d = -1;  // background producer / consumer of the loaded mode
};

/// Host-only queue baselines through one adapter contract (the reference's
/// benchmarks/queue_baselines harness without a GPU): the kiwi ring (this
/// wire format), a head/tail-counter ring of 64-byte slots, a per-slot
/// sequence ring, and a single-word store floor.  Two CPU threads; ping-pong
/// of `iters` round trips (after `warmup`) and a stream of `messages`.
std::vector<BaselineResult> queue_baselines(uint64_t iters, uint64_t warmup, uint64_t messages, uint32_t payload_bytes,
                                            uint64_t capacity, int cpu_a, int cpu_b);
/// The same with every mode's options (idle-poll and loaded-latency included).
std::vector<BaselineResult> queue_baselines(const BaselineOptions& options);

}  // namespace kiwi::bench
