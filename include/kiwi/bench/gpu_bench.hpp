// GPU queue / invoke benchmarks and correctness drivers (host API, no torch).
// Each function launches its kernel, runs the host side of the protocol on the
// calling thread, synchronises, and returns what it measured or received.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace kiwi::bench {

struct RttConfig {
    uint64_t iters = 100000;
    uint64_t warmup = 10000;
    uint32_t payload_bytes = 8;    // request payload (8 B .. 4 KB)
    uint64_t seed = 1;
    int cpu = -1;                  // host thread core (-1: GPU-local core chosen by caller)
    uint64_t capacity = 4096;      // request ring lines
    bool mpsc = false;             // use the MPSC request queue
    uint32_t poll_warps = 1;       // ring replies: warps polling the reply line (staggered)
    bool mailbox = true;           // replies through the mirrored ReplyMailbox (call/return API)
    uint32_t stagger_ns = 200;     // mailbox: delay between the two in-flight polls
    uint32_t initial_delay_ns = 300; // mailbox: (starting) delay before the first poll
    uint32_t pipeline = 1;           // mailbox: polls in flight (1 or 2)
    bool demote = true;              // mailbox: CLDEMOTE each reply line after writing it
    bool adaptive = true;            // mailbox: adapt the delay
    uint64_t timeout_ns = 2000000000ull;
    uint32_t block_threads = 0;      // launch width (0: the warps used; wider blocks idle the extra warps)
};

struct RttResult {
    std::vector<uint64_t> lat_ns;      // per iteration, %globaltimer
    std::vector<uint64_t> lat_cycles;  // per iteration, %clock64
    uint64_t total_ns = 0;             // whole timed loop, %globaltimer
    uint64_t total_cycles = 0;
    uint64_t callbacks = 0;
    uint32_t status = 0;               // kiwi::Status of the device loop
    bool ok = false;                   // every reply matched payload + 1
};

/// GPU -> CPU -> GPU invoke round trip: the kernel invokes a host callback with
/// a seeded payload, the callback replies payload + 1 through an H2D ring.
RttResult invoke_rtt(const RttConfig& cfg);

/// Raw floor: the GPU stores a counter to host memory and polls a host word
/// the CPU sets in reply.  No queue logic.
RttResult pcie_floor(uint64_t iters, uint64_t warmup, int cpu, uint64_t timeout_ns);

/// Store-and-poll protocol variants (see csrc/queue_gpu.cu rtt_lab_kernel).
RttResult rtt_lab(uint64_t iters, uint64_t warmup, uint32_t pollers, uint32_t mirrors, uint32_t stagger_ns,
                  uint32_t fence, uint32_t pipeline, int cpu, uint32_t initial_delay_ns = 0);

/// GPU-producer queue comparators (csrc/queue_baselines_gpu.cu): one driver
/// kernel, one pinned host consumer thread, per-message validation.
struct GpuQueueBaselineOptions {
    std::string queue = "kiwi_spsc";   // kiwi_spsc, kiwi_mpsc, fifo_trigger, proxy_channel, raw_store
    std::string mode = "latency";      // latency, throughput, push_cost
    uint64_t iters = 10000;            // per warp (throughput, push_cost) or timed round trips (latency)
    uint64_t warmup = 1000;            // latency mode
    uint32_t warps = 1;                // producer warps (throughput, push_cost)
    uint64_t capacity = 4096;          // messages the queue holds
    int cpu = -1;                      // consumer thread core (-1: a GPU-local core)
    uint64_t timeout_ns = 2000000000ull;
};

struct GpuQueueBaselineResult {
    std::string queue, mode;
    bool ok = false;                   // every message arrived once, in per-producer order, with its check word
    uint32_t status = 0;               // kiwi::Status of the device side (0 = ok)
    uint64_t messages = 0, bad = 0, order_errors = 0;
    double seconds = 0;                // host wall clock from launch to the last pop
    double cycles_per_push = 0;        // throughput / push_cost: SM cycles per push, mean over warps
    std::vector<uint64_t> lat_ns;      // latency: push -> host pop -> ack seen, per timed iteration
};

GpuQueueBaselineResult gpu_queue_baseline(const GpuQueueBaselineOptions& options);

struct AtomicityResult {
    uint64_t reads = 0;    // 16-byte chunks the host read while the GPU wrote
    uint64_t torn8 = 0;    // 8-byte halves whose two words came from different rounds
    uint64_t tag_ahead = 0;  // of those, halves whose tag word was newer than the data word
    uint64_t split16 = 0;  // chunks whose two halves came from different rounds (allowed)
    uint64_t torn_word = 0;  // 32-bit words whose 16-bit halves disagree (self-checking modes)
    uint64_t torn_nonzero = 0;  // reads that are neither old, new nor zero per word (must be 0)
    bool final_ok = false;
    std::vector<uint64_t> samples;  // the first torn 8-byte halves (H2D: torn words) as read
};
/// GPU rewrites one host line (mode 0: 16-byte stores, 1: 8-byte stores); a host
/// thread classifies every 8-byte half it reads.
AtomicityResult atomicity_test(uint32_t iters, uint32_t mode = 0);
struct ProtocolResult {
    uint64_t rounds = 0;
    uint64_t reads = 0;
    uint64_t torn = 0;          // halves that were neither the old nor the new round
    uint64_t accepted_bad = 0;  // halves with the expected tag but wrong data (must be 0)
    bool ok = false;
    std::vector<uint64_t> samples;
};

/// Ring-reader view of the wire format (format 0) or a {data32, tag32} half
/// (format 1): GPU writes round i, the host waits for it and acknowledges.
ProtocolResult atomicity_protocol_test(uint32_t iters, uint32_t format);

/// Host -> device direction: the host rewrites the line with tagged words
/// (8-byte stores) for `duration_ms`, one GPU warp reads it with 16-byte loads.
AtomicityResult atomicity_h2d_test(uint32_t duration_ms);

struct ThroughputResult {
    uint64_t messages = 0;
    uint64_t device_ns = 0;  // first push to last push (device %globaltimer)
    bool ok = false;
};
/// `endpoints` producer warps invoke a counting callback `msgs_per_endpoint`
/// times each; `threads` native progress threads consume.
ThroughputResult invoke_throughput(uint32_t endpoints, uint32_t threads, uint32_t msgs_per_endpoint,
                                   uint32_t payload_bytes, uint64_t capacity);

struct PushCostResult {
    double cycles_per_push = 0;
    bool ok = false;
};
/// SM cycles one warp spends in push_lanes (ring never full: host drains).
PushCostResult push_cost(uint32_t msgs, uint32_t bytes);

struct GridPollResult {
    uint32_t blocks = 0, pollers = 0;   // pollers = warps of blocks 1.. (lane 0 of each polls)
    double first_observe_p50_ns = 0;    // publish -> first warp saw it (p50 over rounds)
    double last_observe_p50_ns = 0;     // publish -> last warp saw it
    double last_observe_p99_ns = 0;
    double ack_p50_ns = 0;              // publish -> block 0 saw every block's ack
    double ack_p99_ns = 0;
    uint32_t status = 0;
    bool ok = false;
};
/// A grid polling one host-mapped slot that block 0 publishes, then acking
/// through host-mapped lines (the reference's host-mapped grid-poll
/// reproducer); `blocks` must fit on the GPU at once.
GridPollResult grid_poll(uint32_t blocks, uint32_t threads, uint32_t rounds, uint64_t delay_ns, uint64_t timeout_ns);

struct InvokeCostResult {
    double cycles_per_call = 0;  // SM cycles per invoke call (lane-masked: per call of 16 messages)
    uint64_t messages = 0;       // messages the host received
    bool ok = false;
};
/// SM cycles one warp spends per invoke(cb, int32, float, uint64), or per
/// invoke_lane_masked with 16 active lanes; the host drains concurrently.
InvokeCostResult invoke_cost(uint32_t calls, bool lane_masked);

struct PushTestResult {
    uint64_t popped = 0;
    uint64_t mismatches = 0;     // payload / length / metadata errors
    uint64_t order_errors = 0;   // per-warp sequence errors
    uint32_t device_error = 0;   // ErrorRecord code
    std::string first_error;
};

/// Device-to-host push paths.  mode: "global", "lanes", "reg", "lane_masked".
/// sizes: the message sizes to cycle through.  launches > 1 re-launches with the
/// saved SPSC handle.  For MPSC, `warps` producer warps push concurrently.
PushTestResult d2h_push_test(const std::string& mode, bool mpsc, uint64_t capacity,
                             uint32_t warps, uint32_t msgs_per_warp,
                             const std::vector<uint32_t>& sizes, uint32_t launches,
                             uint64_t seed);

/// Host-to-device SPSC: the host pushes `count` messages of the given sizes
/// while one warp pops them into device memory; returns mismatches.
PushTestResult h2d_spsc_test(uint64_t capacity, uint32_t count, const std::vector<uint32_t>& sizes,
                             bool registers, uint32_t notify_interval, uint64_t seed);

/// Host-to-device MPMC: `producers` host threads push, `warps` warps pop.
PushTestResult h2d_mpmc_test(uint64_t slots, uint32_t slot_lines, uint32_t producers,
                             uint32_t msgs_per_producer, uint32_t warps, uint64_t seed);

/// A device wait that nothing satisfies must return kTimeout (not hang).
uint32_t h2d_timeout_test(uint64_t timeout_ns);

struct KernelAttr {
    std::string name;
    int local_bytes;
    int registers;
};
/// Local-memory use of the queue hot-path kernels (must be 0: register resident).
std::vector<KernelAttr> queue_kernel_attributes();

}  // namespace kiwi::bench
