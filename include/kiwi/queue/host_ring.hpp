// Host-side reader and writer of a kiwi::queue ring (see wire.hpp).
//
// RingReader is the host consumer of a device-to-host ring (and, in the
// host-only tests, of a ring a CPU thread writes).  RingWriter is the host
// producer of a host-to-device ring (and the CPU stand-in for a GPU producer).
// Both are plain C++: they compile without CUDA.
//
// Behaviour parity with the reference's host consumer
// (src/queue/chunk_consumer.hpp:97-215 of AMDResearch/kiwi): a message is
// consumed only when every tag of every line it occupies, padding included,
// matches; a corrupt length raises; the consumer position is published after
// every pop so a producer waiting for credit sees it at once.
#pragma once

#include <atomic>
#include <cstring>

#include "kiwi/queue/wire.hpp"

namespace kiwi::queue {

class queue_error : public kiwi::error {
public:
    using kiwi::error::error;
};

namespace host {

inline uint64_t load_half(const void* p) {
    return __atomic_load_n(static_cast<const uint64_t*>(p), __ATOMIC_RELAXED);
}

inline void store_half(void* p, uint64_t v) {
    __atomic_store_n(static_cast<uint64_t*>(p), v, __ATOMIC_RELAXED);
}

/// Hints the core to move the cache line holding `p` to the shared last-level
/// cache (x86 CLDEMOTE), so a device read of it over PCIe does not have to
/// snoop this core's private caches.  Executes as a no-op on CPUs without it.
inline void demote_line(const void* p) {
#if defined(__x86_64__)
    asm volatile("cldemote %0" ::"m"(*static_cast<const volatile char*>(p)));
#else
    (void)p;
#endif
}


inline void cpu_relax() {
#if defined(__x86_64__) || defined(__i386__)
    __builtin_ia32_pause();
#elif defined(__aarch64__)
    asm volatile("yield" ::: "memory");
#endif
}

}  // namespace host

/// Cheap "is a message there?" check: one load of chunk 0's first tag at the
/// consumer position.  A hint only: it can be true while the rest of the
/// message is still in flight (then try_pop returns false).
class HostPollState {
public:
    HostPollState() = default;
    HostPollState(const Chunk* ring, uint64_t capacity, const uint64_t* tail)
        : ring_(ring), mask_(capacity - 1), log2_(log2_pow2(capacity)), tail_(tail) {
        refresh();
    }
    bool ready() const {
        return half_has_tag(host::load_half(word_), expected_);
    }
    void refresh() {
        const uint64_t t = *tail_;
        word_ = &ring_[(t & mask_) * kChunksPerLine].lo;
        expected_ = lap_tag(t, log2_);
    }

private:
    const Chunk* ring_ = nullptr;
    uint64_t mask_ = 0;
    uint32_t log2_ = 0;
    const uint64_t* tail_ = nullptr;
    const uint64_t* word_ = nullptr;
    uint32_t expected_ = 0xffffffffu;
};

class RingReader {
public:
    RingReader() = default;
    /// `published` receives the consumer position (lines) after every pop; the
    /// producer reads it for credit.  It may be null (no producer credit).
    RingReader(Chunk* ring, uint64_t capacity, uint64_t* published, uint64_t start = 0)
        : ring_(ring), capacity_(capacity), mask_(capacity - 1),
          log2_(log2_pow2(capacity)), tail_(start), published_(published) {
        check_capacity(capacity);
        publish();
    }

    /// Pops one whole message into `out` (room for round_up(bytes, 8) bytes,
    /// at most kMaxMessageBytes), or returns false without consuming anything.
    bool try_pop(void* out, uint32_t* metadata, uint32_t* bytes) {
        const uint64_t line0 = tail_;
        const Chunk* c0 = chunk(line0, 0);
        const uint32_t tag0 = lap_tag(line0, log2_);
        const uint64_t h0 = host::load_half(&c0->lo);
        if (!half_has_tag(h0, tag0)) return false;
        const uint64_t h1 = host::load_half(&c0->hi);
        if (!half_has_tag(h1, tag0)) return false;
        const uint32_t len = half_data(h1);
        if (len > kMaxMessageBytes) {
            throw queue_error("kiwi::queue: corrupt message length " + std::to_string(len) +
                              " at line " + std::to_string(line0));
        }
        const uint32_t nchunks = message_chunks(len);
        const uint32_t nlines = message_lines(len);
        if (nlines > capacity_) {
            throw queue_error("kiwi::queue: message of " + std::to_string(len) +
                              " bytes does not fit a ring of " + std::to_string(capacity_) +
                              " lines");
        }
        // The padding chunks of the last line carry no data but are validated
        // too, before any payload is copied: the consumer position published
        // after this pop is the producers' credit, and a padding store still in
        // flight when a line is handed back could land on the next lap's
        // message there (from another producer, on an MPSC ring) and leave it
        // with a stale tag.
        for (uint32_t k = nchunks > 1 ? nchunks : 1; k < nlines * kChunksPerLine; ++k) {
            const uint64_t line = line0 + k / kChunksPerLine;
            const uint32_t tag = lap_tag(line, log2_);
            const Chunk* c = chunk(line, k % kChunksPerLine);
            if (!half_has_tag(host::load_half(&c->lo), tag) || !half_has_tag(host::load_half(&c->hi), tag)) {
                return false;
            }
        }
        uint8_t* dst = static_cast<uint8_t*>(out);
        for (uint32_t k = 1; k < nchunks; ++k) {
            const uint64_t line = line0 + k / kChunksPerLine;
            const uint32_t tag = lap_tag(line, log2_);
            const Chunk* c = chunk(line, k % kChunksPerLine);
            const uint64_t a = host::load_half(&c->lo);
            const uint64_t b = host::load_half(&c->hi);
            if (!half_has_tag(a, tag) || !half_has_tag(b, tag)) return false;
            const uint32_t lo = half_data(a), hi = half_data(b);
            std::memcpy(dst + 8 * (k - 1), &lo, 4);
            std::memcpy(dst + 8 * (k - 1) + 4, &hi, 4);
        }
        if (metadata) *metadata = half_data(h0);
        if (bytes) *bytes = len;
        tail_ = line0 + nlines;
        publish();
        return true;
    }

    HostPollState poll_state() const { return HostPollState(ring_, capacity_, &tail_); }
    uint64_t tail() const { return tail_; }
    uint64_t capacity() const { return capacity_; }

private:
    const Chunk* chunk(uint64_t line, uint32_t c) const {
        return &ring_[(line & mask_) * kChunksPerLine + c];
    }
    void publish() {
        if (published_) __atomic_store_n(published_, tail_, __ATOMIC_RELEASE);
    }

    Chunk* ring_ = nullptr;
    uint64_t capacity_ = 0, mask_ = 0;
    uint32_t log2_ = 0;
    uint64_t tail_ = 0;
    uint64_t* published_ = nullptr;
};

/// Host producer.  Credit comes from the consumer's published position.  A
/// writer starts with credit for `capacity` lines from `start`, i.e. it assumes
/// the consumer is at `start`; a producer that begins elsewhere checks the
/// consumer's position first (MPSCD2HQueue::host_push).
class RingWriter {
public:
    RingWriter() = default;
    RingWriter(Chunk* ring, uint64_t capacity, const uint64_t* consumer_pos, uint64_t start = 0)
        : ring_(ring), capacity_(capacity), mask_(capacity - 1), log2_(log2_pow2(capacity)),
          head_(start), consumer_pos_(consumer_pos), credit_limit_(start + capacity) {
        check_capacity(capacity);
    }

    /// Lines a push of `bytes` would need; throws if the ring can never hold it.
    uint32_t lines_for(uint32_t bytes) const {
        if (bytes > kMaxMessageBytes) {
            throw queue_error("kiwi::queue: message of " + std::to_string(bytes) +
                              " bytes exceeds kMaxMessageBytes");
        }
        const uint32_t n = message_lines(bytes);
        if (n > capacity_) {
            throw queue_error("kiwi::queue: message of " + std::to_string(bytes) +
                              " bytes needs " + std::to_string(n) + " lines; ring has " +
                              std::to_string(capacity_));
        }
        return n;
    }

    bool has_credit(uint32_t nlines) {
        if (head_ + nlines <= credit_limit_) return true;
        if (consumer_pos_) {
            credit_limit_ = __atomic_load_n(consumer_pos_, __ATOMIC_ACQUIRE) + capacity_;
        }
        return head_ + nlines <= credit_limit_;
    }

    /// Writes one message, or returns false (nothing written) if the ring is full.
    bool try_push(const void* payload, uint32_t bytes, uint32_t metadata) {
        const uint32_t nlines = lines_for(bytes);
        if (!has_credit(nlines)) return false;
        write(payload, bytes, metadata, nlines);
        return true;
    }

    /// Writes chunks [first_chunk, last_chunk) of a message at the current
    /// position without advancing it; used by the fault-injection tests to
    /// publish a message in pieces.  Chunk 0 is the header.
    void write_chunks(const void* payload, uint32_t bytes, uint32_t metadata,
                      uint32_t first_chunk, uint32_t last_chunk) const {
        const uint8_t* src = static_cast<const uint8_t*>(payload);
        const uint32_t nchunks = message_chunks(bytes);
        for (uint32_t k = first_chunk; k < last_chunk; ++k) {
            const uint64_t line = head_ + k / kChunksPerLine;
            const uint32_t tag = lap_tag(line, log2_);
            Chunk* c = &ring_[(line & mask_) * kChunksPerLine + k % kChunksPerLine];
            uint32_t lo = 0, hi = 0;
            if (k == 0) {
                lo = metadata;
                hi = bytes;
            } else if (k < nchunks) {
                const uint32_t off = 8 * (k - 1);
                const uint32_t n = bytes - off < 8 ? bytes - off : 8;
                uint8_t w[8] = {0};
                std::memcpy(w, src + off, n);
                std::memcpy(&lo, w, 4);
                std::memcpy(&hi, w + 4, 4);
            }
            host::store_half(&c->lo, pack_half(lo, tag));
            host::store_half(&c->hi, pack_half(hi, tag));
        }
    }

    void advance(uint32_t nlines) { head_ += nlines; }
    uint64_t head() const { return head_; }
    uint64_t capacity() const { return capacity_; }

private:
    void write(const void* payload, uint32_t bytes, uint32_t metadata, uint32_t nlines) {
        // Payload chunks first, header last: a consumer that sees the header has
        // usually got the rest already (each half is self-validating either way).
        write_chunks(payload, bytes, metadata, 1, nlines * kChunksPerLine);
        std::atomic_thread_fence(std::memory_order_release);
        write_chunks(payload, bytes, metadata, 0, 1);
        // The device polls these lines over PCIe: move them to the shared LLC
        // so its reads need not snoop this core's caches (as the reply mailbox).
        for (uint32_t l = 0; l < nlines; ++l) host::demote_line(&ring_[((head_ + l) & mask_) * kChunksPerLine]);
        head_ += nlines;
    }

    Chunk* ring_ = nullptr;
    uint64_t capacity_ = 0, mask_ = 0;
    uint32_t log2_ = 0;
    uint64_t head_ = 0;
    const uint64_t* consumer_pos_ = nullptr;
    uint64_t credit_limit_ = 0;
};

}  // namespace kiwi::queue
