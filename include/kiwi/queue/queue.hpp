// kiwi::queue public host API: the four queue kinds and their owners.
//
// Parity with the reference's public aliases (include/kiwi/queue/queue.hip.hpp:21-41
// and include/kiwi/queue/queue.hpp:51-63 of AMDResearch/kiwi):
//   SPSCD2HQueue  one GPU warp  -> one host thread
//   MPSCD2HQueue  many GPU warps -> one host thread
//   SPSCH2DQueue  one host thread -> one GPU warp
//   MPMCH2DQueue  many host threads -> many GPU warps
// Capacities are in 64-byte lines (slots for MPMC) and must be powers of two.
#pragma once

#include <chrono>

#include <memory>
#include <mutex>

#include "kiwi/queue/handles.cuh"
#include "kiwi/queue/host_memory.hpp"
#include "kiwi/queue/host_ring.hpp"

namespace kiwi::queue {

enum class Direction { kDeviceToHost, kHostToDevice };
enum class Concurrency { kSPSC, kMPSC, kMPMC };

namespace detail {
/// Owns one allocation made through alloc_zeroed().
struct Block {
    void* ptr = nullptr;
    MemKind kind = MemKind::kHost;
    Block() = default;
    Block(size_t bytes, MemKind k) : ptr(alloc_zeroed(bytes, k)), kind(k) {}
    ~Block() { free_memory(ptr, kind); }
    Block(const Block&) = delete;
    Block& operator=(const Block&) = delete;
    template <typename T>
    T* as() const { return static_cast<T*>(ptr); }
    template <typename T>
    T* dev() const { return static_cast<T*>(device_address(ptr, kind)); }
};
}  // namespace detail

/// Common state of the two device-to-host rings.
class D2HRingBase {
public:
    D2HRingBase(uint64_t capacity, MemKind kind)
        : capacity_(capacity), kind_(kind),
          ring_((check_capacity(capacity), capacity * kLineBytes), kind),
          pos_(sizeof(uint64_t), kind), err_(sizeof(ErrorRecord), kind),
          reader_(ring_.as<Chunk>(), capacity, pos_.as<uint64_t>()) {}

    /// Pops one whole message; see RingReader::try_pop.
    bool try_pop(void* out, uint32_t* metadata, uint32_t* bytes) {
        return reader_.try_pop(out, metadata, bytes);
    }
    HostPollState host_poll_state() const { return reader_.poll_state(); }
    uint64_t capacity() const { return capacity_; }
    /// The consumer's published position (safe to read from any thread).
    uint64_t consumer_position() const { return __atomic_load_n(pos_.as<const uint64_t>(), __ATOMIC_ACQUIRE); }
    MemKind memory_kind() const { return kind_; }

    /// Error recorded by device code (code 0 = none).
    ErrorRecord error() const {
        ErrorRecord r;
        const volatile ErrorRecord* e = err_.as<volatile ErrorRecord>();
        r.code = e->code;
        r.site = e->site;
        r.rank = e->rank;
        r.info = e->info;
        return r;
    }
    void clear_error() { *err_.as<volatile uint32_t>() = 0; }

    /// CPU stand-in producer positioned at the consumer (host-only tests).
    /// Reads the position the consumer publishes (not its private cursor), so
    /// it may be called while progress threads pop; call it when no other
    /// producer has messages in flight, since it starts where they would be.
    RingWriter host_writer_any() const {
        return RingWriter(ring_.as<Chunk>(), capacity_, pos_.as<const uint64_t>(), consumer_position());
    }

    /// Host pointers, for CPU stand-in producers in tests and benchmarks.
    Chunk* ring_host() const { return ring_.as<Chunk>(); }
    const uint64_t* consumer_pos_host() const { return pos_.as<uint64_t>(); }

protected:
    uint64_t capacity_;
    MemKind kind_;
    detail::Block ring_;
    detail::Block pos_;
    detail::Block err_;
    RingReader reader_;
};

class SPSCD2HQueue : public D2HRingBase {
public:
    using DeviceHandle = SpscD2HHandle;
    explicit SPSCD2HQueue(uint64_t capacity, MemKind kind = default_host_kind())
        : D2HRingBase(capacity, kind) {}

    /// A producer handle starting at the consumer position.  The queue must be
    /// drained (every pushed message popped) when it is called, because the
    /// SPSC producer position lives only in the handle.
    DeviceHandle device_handle() const {
        DeviceHandle h{};
        h.ring = ring_.dev<Chunk>();
        h.consumer_pos = pos_.dev<const uint64_t>();
        h.err = err_.dev<ErrorRecord>();
        h.head = reader_.tail();
        h.credit_limit = reader_.tail() + capacity_;
        h.log2cap = log2_pow2(capacity_);
        return h;
    }

    /// CPU stand-in producer positioned like device_handle().
    RingWriter host_writer() const { return host_writer_any(); }
};

class MPSCD2HQueue : public D2HRingBase {
public:
    using DeviceHandle = MpscD2HHandle;
    explicit MPSCD2HQueue(uint64_t capacity, MemKind kind = default_host_kind(),
                          MemKind counter_kind = MemKind::kDevice)
        : D2HRingBase(capacity, kind),
          claim_(sizeof(unsigned long long),
                 kind == MemKind::kHost ? MemKind::kHost : counter_kind) {}

    /// Handles may be copied to any number of warps and used concurrently.
    DeviceHandle device_handle(uint64_t timeout_ns = kDefaultTimeoutNs) const {
        DeviceHandle h{};
        h.ring = ring_.dev<Chunk>();
        h.consumer_pos = pos_.dev<const uint64_t>();
        h.err = err_.dev<ErrorRecord>();
        h.claim = claim_.dev<unsigned long long>();
        h.credit_limit = reader_.tail() + capacity_;
        h.timeout_ns = timeout_ns;
        h.log2cap = log2_pow2(capacity_);
        return h;
    }

    /// CPU stand-in for the device producers (host-only queues: tests and
    /// host-side stress).  The same protocol as MpscD2HHandle: claim the
    /// message's lines with a fetch-add on the producer counter, wait for the
    /// consumer's credit, then write the message there (header last).
    /// Thread-safe.  A claimed range must be written or the consumer stalls at
    /// it, so a credit wait that runs out throws instead of returning.
    void host_push(const void* payload, uint32_t bytes, uint32_t metadata, double timeout_s = 10.0) {
        if (ring_.kind != MemKind::kHost) throw kiwi::error("host_push needs a host-only (MemKind::kHost) queue");
        if (bytes > kMaxMessageBytes || message_lines(bytes) > capacity_) {
            throw kiwi::error("kiwi::queue: host_push of " + std::to_string(bytes) + " bytes does not fit");
        }
        const uint32_t nlines = message_lines(bytes);
        const uint64_t base = __atomic_fetch_add(claim_.as<unsigned long long>(), nlines, __ATOMIC_RELAXED);
        // Credit from the consumer's published position (a writer constructed at
        // `base` would assume the ring is empty there).
        const auto deadline = std::chrono::steady_clock::now() + std::chrono::duration<double>(timeout_s);
        while (base + nlines > consumer_position() + capacity_) {
            if (std::chrono::steady_clock::now() > deadline) {
                throw kiwi::error("kiwi::queue: host_push waited too long for consumer credit");
            }
            host::cpu_relax();
        }
        RingWriter w(ring_.as<Chunk>(), capacity_, pos_.as<const uint64_t>(), base);
        if (!w.try_push(payload, bytes, metadata)) throw kiwi::error("kiwi::queue: host_push lost its credit");
    }

private:
    detail::Block claim_;
};

class SPSCH2DQueue {
public:
    /// `notify_interval` = lines the device consumes before it publishes its
    /// position (1 = every pop).  A larger interval saves PCIe writes; the
    /// consumer must then call flush_consumer_index() before it exits.
    explicit SPSCH2DQueue(uint64_t capacity, MemKind kind = default_host_kind(),
                          uint32_t notify_interval = 1)
        : capacity_(capacity), notify_(notify_interval),
          ring_((check_capacity(capacity), capacity * kLineBytes), kind),
          pos_(sizeof(uint64_t), kind), err_(sizeof(ErrorRecord), kind),
          writer_(ring_.as<Chunk>(), capacity, pos_.as<const uint64_t>()) {
        if (notify_interval == 0 || notify_interval > capacity) {
            throw kiwi::error("kiwi::queue: notify_interval must be in [1, capacity]");
        }
    }

    using DeviceHandle = SpscH2DHandle;
    DeviceHandle device_handle() const {
        DeviceHandle h{};
        h.ring = ring_.dev<const Chunk>();
        h.consumer_pos = pos_.dev<uint64_t>();
        h.err = err_.dev<ErrorRecord>();
        h.tail = *pos_.as<volatile uint64_t>();
        h.published = h.tail;
        h.log2cap = log2_pow2(capacity_);
        h.notify_interval = notify_;
        return h;
    }

    /// Host producer; returns false (nothing written) when the ring is full.
    bool try_push(const void* payload, uint32_t bytes, uint32_t metadata = 0) {
        return writer_.try_push(payload, bytes, metadata);
    }
    uint64_t capacity() const { return capacity_; }
    uint64_t producer_position() const { return writer_.head(); }
    uint64_t consumer_position() const { return *pos_.as<volatile uint64_t>(); }
    Chunk* ring_host() const { return ring_.as<Chunk>(); }
    uint64_t* consumer_pos_host() const { return pos_.as<uint64_t>(); }
    ErrorRecord error() const { return *err_.as<ErrorRecord>(); }

private:
    uint64_t capacity_;
    uint32_t notify_;
    detail::Block ring_;
    detail::Block pos_;
    detail::Block err_;
    RingWriter writer_;
};

class MPMCH2DQueue {
public:
    /// `slots` fixed slots of `slot_lines` lines (payload (4*slot_lines-1)*8 bytes;
    /// the default 2 lines carry 56 bytes).
    explicit MPMCH2DQueue(uint64_t slots, uint32_t slot_lines = 2,
                          MemKind kind = default_host_kind())
        : slots_(slots), slot_lines_(slot_lines),
          ring_((check_capacity(slots), slots * slot_lines * kLineBytes), kind),
          acks_(slots * sizeof(uint32_t), kind), err_(sizeof(ErrorRecord), kind),
          claim_(sizeof(unsigned long long), kind == MemKind::kHost ? MemKind::kHost : MemKind::kDevice),
          log2_(log2_pow2(slots)) {
        if (slot_lines == 0 || slot_lines > 8) {
            throw kiwi::error("kiwi::queue: MPMC slot_lines must be in [1, 8]");
        }
    }

    using DeviceHandle = MpmcH2DHandle;
    DeviceHandle device_handle() const {
        DeviceHandle h{};
        h.ring = ring_.dev<const Chunk>();
        h.claim = claim_.dev<unsigned long long>();
        h.acks = acks_.dev<uint32_t>();
        h.err = err_.dev<ErrorRecord>();
        h.log2slots = log2_;
        h.slot_lines = slot_lines_;
        return h;
    }

    uint32_t slot_payload_bytes() const { return (slot_lines_ * kChunksPerLine - 1) * 8; }

    /// Thread-safe host producer.  Returns false if the next slot is still held
    /// by an earlier lap (queue full).
    bool try_push(const void* payload, uint32_t bytes, uint32_t metadata = 0) {
        if (bytes > slot_payload_bytes()) {
            throw queue_error("kiwi::queue: MPMC message of " + std::to_string(bytes) +
                              " bytes exceeds the slot payload of " +
                              std::to_string(slot_payload_bytes()));
        }
        uint64_t pos = __atomic_load_n(&head_, __ATOMIC_RELAXED);
        while (true) {
            const uint64_t slot = pos & (slots_ - 1);
            const uint32_t lap = static_cast<uint32_t>(pos >> log2_);
            const uint32_t acked = __atomic_load_n(&acks_.as<uint32_t>()[slot], __ATOMIC_ACQUIRE);
            if (acked != lap) return false;
            if (__atomic_compare_exchange_n(&head_, &pos, pos + 1, false, __ATOMIC_ACQ_REL,
                                            __ATOMIC_RELAXED)) {
                write_slot(slot, wire_tag(lap), payload, bytes, metadata);
                return true;
            }
        }
    }

    /// CPU stand-in for the device consumers (host-only queues: tests and
    /// host-side stress).  The same protocol as MpmcH2DHandle::try_pop: read
    /// the claimed position's slot, check every word's lap tag, take the slot
    /// with a CAS on the claim counter, copy the payload, then ack the slot so
    /// producers can reuse it.  Thread-safe; false when the next slot is empty
    /// or another consumer took it first.
    bool host_try_pop(void* out, uint32_t* metadata, uint32_t* bytes) {
        if (ring_.kind != MemKind::kHost) throw kiwi::error("host_try_pop needs a host-only (MemKind::kHost) queue");
        auto* claim = claim_.as<unsigned long long>();
        const uint64_t pos = __atomic_load_n(claim, __ATOMIC_ACQUIRE);
        const uint64_t slot = pos & (slots_ - 1);
        const uint32_t lap = static_cast<uint32_t>(pos >> log2_);
        const uint32_t tag = wire_tag(lap);
        const uint32_t total = slot_lines_ * kChunksPerLine;
        const Chunk* base = ring_.as<Chunk>() + slot * total;
        uint32_t lo[kChunksPerLine * 8], hi[kChunksPerLine * 8];
        for (uint32_t k = 0; k < total; ++k) {
            const uint64_t a = host::load_half(&base[k].lo);
            const uint64_t b = host::load_half(&base[k].hi);
            if (!half_has_tag(a, tag) || !half_has_tag(b, tag)) return false;
            lo[k] = half_data(a);
            hi[k] = half_data(b);
        }
        unsigned long long expect = pos;
        if (!__atomic_compare_exchange_n(claim, &expect, pos + 1, false, __ATOMIC_ACQ_REL, __ATOMIC_RELAXED)) {
            return false;
        }
        const uint32_t len = hi[0];
        if (metadata) *metadata = lo[0];
        if (len > slot_payload_bytes()) {
            __atomic_store_n(&acks_.as<uint32_t>()[slot], lap + 1, __ATOMIC_RELEASE);
            throw queue_error("kiwi::queue: MPMC slot holds a length of " + std::to_string(len) + " bytes");
        }
        uint8_t* dst = static_cast<uint8_t*>(out);
        for (uint32_t k = 1; 8 * (k - 1) < len; ++k) {
            uint8_t w[8];
            std::memcpy(w, &lo[k], 4);
            std::memcpy(w + 4, &hi[k], 4);
            const uint32_t off = 8 * (k - 1);
            std::memcpy(dst + off, w, len - off < 8 ? len - off : 8);
        }
        if (bytes) *bytes = len;
        __atomic_store_n(&acks_.as<uint32_t>()[slot], lap + 1, __ATOMIC_RELEASE);
        return true;
    }

    uint64_t slots() const { return slots_; }
    uint64_t producer_position() const { return __atomic_load_n(&head_, __ATOMIC_RELAXED); }
    ErrorRecord error() const { return *err_.as<ErrorRecord>(); }

private:
    void write_slot(uint64_t slot, uint32_t tag, const void* payload, uint32_t bytes,
                    uint32_t metadata) {
        Chunk* base = ring_.as<Chunk>() + slot * slot_lines_ * kChunksPerLine;
        const uint8_t* src = static_cast<const uint8_t*>(payload);
        const uint32_t total = slot_lines_ * kChunksPerLine;
        const uint32_t nchunks = message_chunks(bytes);
        for (uint32_t k = total; k-- > 0;) {  // header (chunk 0) last
            uint32_t lo = 0, hi = 0;
            if (k == 0) {
                lo = metadata;
                hi = bytes;
            } else if (k < nchunks) {
                uint8_t w[8] = {0};
                const uint32_t off = 8 * (k - 1);
                std::memcpy(w, src + off, bytes - off < 8 ? bytes - off : 8);
                std::memcpy(&lo, w, 4);
                std::memcpy(&hi, w + 4, 4);
            }
            host::store_half(&base[k].lo, pack_half(lo, tag));
            host::store_half(&base[k].hi, pack_half(hi, tag));
            if (k == 1) std::atomic_thread_fence(std::memory_order_release);
        }
        for (uint32_t l = 0; l < slot_lines_; ++l) host::demote_line(&base[l * kChunksPerLine]);
    }

    uint64_t slots_;
    uint32_t slot_lines_;
    detail::Block ring_;
    detail::Block acks_;
    detail::Block err_;
    detail::Block claim_;
    uint32_t log2_;
    alignas(64) uint64_t head_ = 0;
};

/// Queue<Direction, Concurrency> selector, as in the reference's template.
template <Direction D, Concurrency C>
struct QueueSelect;
template <>
struct QueueSelect<Direction::kDeviceToHost, Concurrency::kSPSC> { using type = SPSCD2HQueue; };
template <>
struct QueueSelect<Direction::kDeviceToHost, Concurrency::kMPSC> { using type = MPSCD2HQueue; };
template <>
struct QueueSelect<Direction::kHostToDevice, Concurrency::kSPSC> { using type = SPSCH2DQueue; };
template <>
struct QueueSelect<Direction::kHostToDevice, Concurrency::kMPMC> { using type = MPMCH2DQueue; };
template <Direction D, Concurrency C>
using Queue = typename QueueSelect<D, C>::type;

}  // namespace kiwi::queue
