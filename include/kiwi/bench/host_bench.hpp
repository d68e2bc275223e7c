// Host-only queue benchmarks (no GPU needed).
#pragma once

#include <cstdint>
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

}  // namespace kiwi::bench
