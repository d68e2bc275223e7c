// Host-only queue baselines behind one adapter contract (the counterpart of
// the reference's benchmarks/queue_baselines harness, qb_common.hpp's
// adapter contract, run without a GPU).  Every adapter is single-producer /
// single-consumer in plain host memory:
//
//   try_push(payload, bytes, meta)   producer thread only; false when full
//   try_pop(out, &meta, &bytes)      consumer thread only; false when empty
//
//   kiwi_ring   this repository's ring (tagged words in 64-byte lines, the
//               consumer validates tags; no index read on the fast path)
//   head_tail   64-byte slots + producer head / consumer tail counters on
//               their own cache lines (the index-publishing FIFO style)
//   seq_slot    64-byte slots each carrying a sequence word that the
//               producer release-stores after the payload (Vyukov SPSC)
//   raw_word    one 8-byte word per direction holding a counter: the floor
//               of any queue (payload limited to the counter itself)
//
// Modes (the reference's latency, throughput, idle-poll and loaded-latency,
// benchmarks/queue_baselines/README.md:96-104): ping-pong round trip, one-way
// stream, the cost of polling an empty queue, and the ping-pong again while a
// second pair of threads streams through another instance of the same queue.
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstring>
#include <memory>
#include <thread>
#include <vector>

#include "kiwi/bench/host_bench.hpp"
#include "kiwi/queue/host_ring.hpp"
#include "kiwi/queue/queue.hpp"
#include "kiwi/topology.hpp"

namespace kiwi::bench {

namespace {

inline uint64_t now_ns() {
    return static_cast<uint64_t>(
        std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now().time_since_epoch())
            .count());
}

constexpr uint32_t kSlotPayload = 48;  // 64-byte slots minus an 16-byte header

class KiwiRing {
public:
    explicit KiwiRing(uint64_t cap) : q_(cap, queue::MemKind::kHost), w_(q_.host_writer()) {}
    static const char* name() { return "kiwi_ring"; }
    static uint32_t max_payload() { return queue::kMaxMessageBytes; }
    bool try_push(const void* p, uint32_t n, uint32_t meta) { return w_.try_push(p, n, meta); }
    bool try_pop(void* out, uint32_t* meta, uint32_t* n) { return q_.try_pop(out, meta, n); }

private:
    queue::SPSCD2HQueue q_;              // consumer state
    alignas(64) queue::RingWriter w_;    // producer state on its own cache lines
    char pad_[64] = {};
};

struct alignas(64) Slot {
    std::atomic<uint64_t> seq;  // seq_slot only
    uint32_t meta;
    uint32_t bytes;
    uint8_t payload[kSlotPayload];
};
static_assert(sizeof(Slot) == 64, "one cache line per slot");

class HeadTail {
public:
    explicit HeadTail(uint64_t cap) : cap_(cap), slots_(new Slot[cap]) {}
    static const char* name() { return "head_tail"; }
    static uint32_t max_payload() { return kSlotPayload; }
    bool try_push(const void* p, uint32_t n, uint32_t meta) {
        const uint64_t h = head_.v.load(std::memory_order_relaxed);
        if (h - tail_cache_ >= cap_) {
            tail_cache_ = tail_.v.load(std::memory_order_acquire);
            if (h - tail_cache_ >= cap_) return false;
        }
        Slot& s = slots_[h % cap_];
        s.meta = meta;
        s.bytes = n;
        std::memcpy(s.payload, p, n);
        head_.v.store(h + 1, std::memory_order_release);
        return true;
    }
    bool try_pop(void* out, uint32_t* meta, uint32_t* n) {
        const uint64_t t = tail_.v.load(std::memory_order_relaxed);
        if (t == head_cache_) {
            head_cache_ = head_.v.load(std::memory_order_acquire);
            if (t == head_cache_) return false;
        }
        const Slot& s = slots_[t % cap_];
        *meta = s.meta;
        *n = s.bytes;
        std::memcpy(out, s.payload, s.bytes);
        tail_.v.store(t + 1, std::memory_order_release);
        return true;
    }

private:
    struct alignas(64) Index {
        std::atomic<uint64_t> v{0};
    };
    uint64_t cap_;
    std::unique_ptr<Slot[]> slots_;
    Index head_, tail_;
    alignas(64) uint64_t tail_cache_ = 0;  // producer's view
    alignas(64) uint64_t head_cache_ = 0;  // consumer's view
};

class SeqSlot {
public:
    explicit SeqSlot(uint64_t cap) : cap_(cap), slots_(new Slot[cap]) {
        for (uint64_t i = 0; i < cap; ++i) slots_[i].seq.store(i, std::memory_order_relaxed);
    }
    static const char* name() { return "seq_slot"; }
    static uint32_t max_payload() { return kSlotPayload; }
    bool try_push(const void* p, uint32_t n, uint32_t meta) {
        Slot& s = slots_[head_ % cap_];
        if (s.seq.load(std::memory_order_acquire) != head_) return false;
        s.meta = meta;
        s.bytes = n;
        std::memcpy(s.payload, p, n);
        s.seq.store(head_ + 1, std::memory_order_release);
        ++head_;
        return true;
    }
    bool try_pop(void* out, uint32_t* meta, uint32_t* n) {
        Slot& s = slots_[tail_ % cap_];
        if (s.seq.load(std::memory_order_acquire) != tail_ + 1) return false;
        *meta = s.meta;
        *n = s.bytes;
        std::memcpy(out, s.payload, s.bytes);
        s.seq.store(tail_ + cap_, std::memory_order_release);
        ++tail_;
        return true;
    }

private:
    uint64_t cap_;
    std::unique_ptr<Slot[]> slots_;
    alignas(64) uint64_t head_ = 0;
    alignas(64) uint64_t tail_ = 0;
};

/// One word per direction: the producer stores ++count (the 8-byte payload is
/// the count's own value); the consumer waits for the next count.
class RawWord {
public:
    explicit RawWord(uint64_t) {}
    static const char* name() { return "raw_word"; }
    static uint32_t max_payload() { return 8; }
    bool try_push(const void*, uint32_t, uint32_t) {
        if (sent_ != acked_.v.load(std::memory_order_acquire)) return false;  // one in flight
        word_.v.store(++sent_, std::memory_order_release);
        return true;
    }
    bool try_pop(void* out, uint32_t* meta, uint32_t* n) {
        const uint64_t v = word_.v.load(std::memory_order_acquire);
        if (v == seen_) return false;
        seen_ = v;
        std::memcpy(out, &v, 8);
        *meta = static_cast<uint32_t>(v - 1);
        *n = 8;
        acked_.v.store(v, std::memory_order_release);
        return true;
    }

private:
    struct alignas(64) W {
        std::atomic<uint64_t> v{0};
    };
    W word_, acked_;
    alignas(64) uint64_t sent_ = 0;
    alignas(64) uint64_t seen_ = 0;
};

/// Ping-pong of `iters` round trips (after `warmup`) over two A queues between
/// the calling thread (cpu_a) and a second thread (cpu_b).  Returns whether
/// order and payloads checked out; fills p50 / p99 in ns.
template <typename A>
bool pingpong(uint64_t iters, uint64_t warmup, uint32_t n, uint64_t cap, int cpu_a, int cpu_b, double* p50,
              double* p99) {
    const bool raw = std::strcmp(A::name(), "raw_word") == 0;
    A a2b(cap), b2a(cap);
    const uint64_t total = iters + warmup;
    std::vector<uint64_t> lat(iters);
    std::atomic<bool> b_ok{true};
    std::thread tb([&] {
        if (cpu_b >= 0) topology::bind_current_thread({cpu_b});
        alignas(64) uint8_t buf[queue::kMaxMessageBytes];
        for (uint64_t i = 0; i < total; ++i) {
            uint32_t meta = 0, bytes = 0;
            while (!a2b.try_pop(buf, &meta, &bytes)) queue::host::cpu_relax();
            if (meta != static_cast<uint32_t>(i)) b_ok = false;
            while (!b2a.try_push(buf, bytes, meta)) queue::host::cpu_relax();
        }
    });
    if (cpu_a >= 0) topology::bind_current_thread({cpu_a});
    alignas(64) uint8_t msg[queue::kMaxMessageBytes] = {0};
    alignas(64) uint8_t buf[queue::kMaxMessageBytes];
    uint64_t state = 0x9E3779B97F4A7C15ull;
    bool ok = true;
    for (uint64_t i = 0; i < total; ++i) {
        const uint64_t v = xorshift64(state);
        std::memcpy(msg, &v, 8);
        const uint64_t t0 = now_ns();
        while (!a2b.try_push(msg, n, static_cast<uint32_t>(i))) queue::host::cpu_relax();
        uint32_t meta = 0, bytes = 0;
        while (!b2a.try_pop(buf, &meta, &bytes)) queue::host::cpu_relax();
        const uint64_t t1 = now_ns();
        uint64_t back;
        std::memcpy(&back, buf, 8);
        if (meta != static_cast<uint32_t>(i) || (!raw && back != v)) ok = false;
        if (i >= warmup) lat[i - warmup] = t1 - t0;
    }
    tb.join();
    std::sort(lat.begin(), lat.end());
    if (!lat.empty()) {
        *p50 = static_cast<double>(lat[lat.size() / 2]);
        *p99 = static_cast<double>(lat[std::min(lat.size() - 1, lat.size() * 99 / 100)]);
    }
    return ok && b_ok;
}

template <typename A>
BaselineResult run_one(const BaselineOptions& o) {
    BaselineResult r;
    r.name = A::name();
    const uint32_t n = std::min<uint32_t>(std::max<uint32_t>(o.payload_bytes, 8), A::max_payload());
    const bool raw = std::strcmp(A::name(), "raw_word") == 0;
    r.ok = pingpong<A>(o.iters, o.warmup, n, o.capacity, o.cpu_a, o.cpu_b, &r.p50_ns, &r.p99_ns);
    // One-way stream.
    {
        A q(o.capacity);
        uint64_t got_sum = 0;
        bool order = true;
        std::thread tb([&] {
            if (o.cpu_b >= 0) topology::bind_current_thread({o.cpu_b});
            alignas(64) uint8_t buf[queue::kMaxMessageBytes];
            for (uint64_t i = 0; i < o.messages; ++i) {
                uint32_t meta = 0, bytes = 0;
                while (!q.try_pop(buf, &meta, &bytes)) queue::host::cpu_relax();
                uint64_t v;
                std::memcpy(&v, buf, 8);
                got_sum += v;
                if (meta != static_cast<uint32_t>(i)) order = false;
            }
        });
        if (o.cpu_a >= 0) topology::bind_current_thread({o.cpu_a});
        alignas(64) uint8_t msg[queue::kMaxMessageBytes] = {0};
        uint64_t state = 0x243F6A8885A308D3ull, sum = 0;
        const uint64_t t0 = now_ns();
        for (uint64_t i = 0; i < o.messages; ++i) {
            const uint64_t v = raw ? i + 1 : xorshift64(state);
            std::memcpy(msg, &v, 8);
            sum += v;
            while (!q.try_push(msg, n, static_cast<uint32_t>(i))) queue::host::cpu_relax();
        }
        tb.join();
        const uint64_t dt = now_ns() - t0;
        r.msgs_per_s = dt ? static_cast<double>(o.messages) / (static_cast<double>(dt) / 1e9) : 0.0;
        r.ok = r.ok && order && got_sum == sum;
    }
    // Idle poll: what one check of an empty queue costs the consumer.
    if (o.idle_polls) {
        A q(o.capacity);
        alignas(64) uint8_t buf[queue::kMaxMessageBytes];
        uint32_t meta = 0, bytes = 0;
        uint64_t hits = 0;
        const uint64_t t0 = now_ns();
        for (uint64_t i = 0; i < o.idle_polls; ++i) hits += q.try_pop(buf, &meta, &bytes) ? 1 : 0;
        r.idle_poll_ns = static_cast<double>(now_ns() - t0) / static_cast<double>(o.idle_polls);
        r.ok = r.ok && hits == 0;
    }
    // Loaded latency: the ping-pong again while two more threads stream
    // through another instance of the same queue (cpu_c produces, cpu_d
    // consumes), sharing caches, memory bandwidth and the scheduler with it.
    if (o.loaded) {
        A bg(o.capacity);
        std::atomic<bool> stop{false};
        std::atomic<uint64_t> streamed{0};
        std::thread prod([&] {
            if (o.cpu_c >= 0) topology::bind_current_thread({o.cpu_c});
            alignas(64) uint8_t msg[queue::kMaxMessageBytes] = {0};
            uint32_t i = 0;
            while (!stop.load(std::memory_order_relaxed)) {
                if (bg.try_push(msg, n, i)) ++i;
                else queue::host::cpu_relax();
            }
        });
        std::thread cons([&] {
            if (o.cpu_d >= 0) topology::bind_current_thread({o.cpu_d});
            alignas(64) uint8_t buf[queue::kMaxMessageBytes];
            uint64_t got = 0;
            while (!stop.load(std::memory_order_relaxed)) {
                uint32_t meta = 0, bytes = 0;
                if (bg.try_pop(buf, &meta, &bytes)) ++got;
                else queue::host::cpu_relax();
            }
            streamed.store(got);
        });
        const uint64_t t0 = now_ns();
        const bool ok = pingpong<A>(o.iters, o.warmup, n, o.capacity, o.cpu_a, o.cpu_b, &r.loaded_p50_ns,
                                    &r.loaded_p99_ns);
        const uint64_t dt = now_ns() - t0;
        stop.store(true);
        prod.join();
        cons.join();
        r.loaded_bg_msgs_per_s = dt ? static_cast<double>(streamed.load()) / (static_cast<double>(dt) / 1e9) : 0.0;
        r.ok = r.ok && ok;
    }
    return r;
}

}  // namespace

std::vector<BaselineResult> queue_baselines(const BaselineOptions& o) {
    if (!is_pow2(o.capacity)) throw kiwi::error("queue_baselines: capacity must be a power of two");
    std::vector<BaselineResult> out;
    out.push_back(run_one<KiwiRing>(o));
    out.push_back(run_one<HeadTail>(o));
    out.push_back(run_one<SeqSlot>(o));
    out.push_back(run_one<RawWord>(o));
    return out;
}

std::vector<BaselineResult> queue_baselines(uint64_t iters, uint64_t warmup, uint64_t messages, uint32_t payload_bytes,
                                            uint64_t capacity, int cpu_a, int cpu_b) {
    BaselineOptions o;
    o.iters = iters;
    o.warmup = warmup;
    o.messages = messages;
    o.payload_bytes = payload_bytes;
    o.capacity = capacity;
    o.cpu_a = cpu_a;
    o.cpu_b = cpu_b;
    return queue_baselines(o);
}

}  // namespace kiwi::bench
