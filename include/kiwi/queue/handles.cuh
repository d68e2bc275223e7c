// Device-side queue handles.  Every operation is warp-collective: all 32 lanes
// of one warp call it from converged code with the same arguments (except the
// per-lane arguments of push_lanes / push_lane_masked).
//
// Behaviour parity with the reference's device queues (AMDResearch/kiwi):
//   SpscD2H  <- include/kiwi/queue/device_to_host_queue.hip.hpp:46-232
//   MpscD2H  <- include/kiwi/queue/mpsc_device_to_host_queue.hip.hpp:68-229
//   SpscH2D  <- include/kiwi/queue/host_to_device_queue.hip.hpp:43-204
//   MpmcH2D  <- include/kiwi/queue/mpmc_host_to_device_queue.hip.hpp:58-277
// The reference is wave64 (lane c stores chunk c).  Here a 32-lane warp
// stores chunks lane, lane+32, ... so a 4 KB message takes 17 stores per lane;
// each store is one st.volatile.global.v4 of a whole chunk, and the lanes of a
// line store together, so every line leaves the GPU as one 64-byte write.
//
// Nothing here traps.  A message that can never fit is dropped and recorded in
// the queue's ErrorRecord (host memory); bounded waits record kTimeout.
#pragma once

#include <type_traits>
#include <utility>

#include "kiwi/queue/wire.hpp"
#if defined(__CUDACC__)
#include "kiwi/ptx.cuh"
#endif

namespace kiwi::queue {

/// Default bound for device waits inside queue operations (2 s).
inline constexpr uint64_t kDefaultTimeoutNs = 2000000000ull;

#if defined(__CUDACC__)
namespace dev {

KIWI_DEV void report(ErrorRecord* err, Status code, uint32_t site, uint32_t info) {
    if (err == nullptr) return;
    if (ptx::lane_id() == 0) {
        ptx::st_volatile_u32(&err->site, site);
        ptx::st_volatile_u32(&err->rank, blockIdx.x);
        ptx::st_volatile_u32(&err->info, info);
        ptx::fence_sys();
        ptx::st_volatile_u32(&err->code, static_cast<uint32_t>(code));
    }
}

/// Stores one chunk {lo, hi} with tag `tag` (one 16-byte store).
KIWI_DEV void store_chunk(Chunk* p, uint32_t lo, uint32_t hi, uint32_t tag) {
    ptx::st_volatile_v4(p, tagged_word(lo, tag), tagged_word(lo >> 16, tag), tagged_word(hi, tag),
                        tagged_word(hi >> 16, tag));
}

/// A chunk loaded with one 16-byte load carries `tag` in all four words.
KIWI_DEV bool chunk_ok(const uint4& v, uint32_t tag) { return words_have_tag(v.x, v.y, v.z, v.w, tag); }
KIWI_DEV uint32_t chunk_lo(const uint4& v) { return join_words(v.x, v.y); }
KIWI_DEV uint32_t chunk_hi(const uint4& v) { return join_words(v.z, v.w); }

/// Writes one message at line `head`.  `word(i)` returns payload word i (8
/// bytes) for the calling lane; it is called only for the lane's own chunks.
template <typename WordFn>
KIWI_DEV void write_message(Chunk* ring, uint32_t log2cap, uint64_t head, uint32_t bytes,
                            uint32_t metadata, WordFn&& word) {
    const uint32_t lane = ptx::lane_id();
    const uint32_t nchunks = message_chunks(bytes);
    const uint32_t total = message_lines(bytes) * kChunksPerLine;
    const uint64_t mask = (uint64_t{1} << log2cap) - 1;
    for (uint32_t k = lane; k < total; k += kWarpSize) {
        const uint64_t line = head + k / kChunksPerLine;
        const uint32_t tag = lap_tag(line, log2cap);
        uint32_t lo = 0, hi = 0;
        if (k == 0) {
            lo = metadata;
            hi = bytes;
        } else if (k < nchunks) {
            const uint64_t w = word(k - 1);
            lo = static_cast<uint32_t>(w);
            hi = static_cast<uint32_t>(w >> 32);
        }
        dev::store_chunk(&ring[(line & mask) * kChunksPerLine + (k & 3u)], lo, hi, tag);
    }
}

template <typename T, typename = void>
struct has_word_array : std::false_type {};
template <typename T>
struct has_word_array<T, std::void_t<decltype(std::declval<const T&>().w[0])>>
    : std::is_same<std::decay_t<decltype(std::declval<const T&>().w[0])>, uint64_t> {};

/// Selects 8-byte word `i` of a register-resident object (all lanes hold it).
template <typename T>
KIWI_DEV uint64_t select_word(const T& msg, uint32_t i) {
    if constexpr (has_word_array<T>::value) {
        constexpr uint32_t kW = sizeof(T) / 8;
        uint64_t out = 0;
#pragma unroll
        for (uint32_t w = 0; w < kW; ++w) out = (w == i) ? msg.w[w] : out;
        return out;
    } else {
        // Assemble each word from pieces at constant offsets (fully unrolled),
        // so even large byte structs stay in registers.
        constexpr uint32_t kWords = (sizeof(T) + 7) / 8;
        constexpr uint32_t kPiece = (alignof(T) >= 4 && sizeof(T) % 4 == 0) ? 4 : 1;
        const char* base = reinterpret_cast<const char*>(&msg);
        uint64_t out = 0;
#pragma unroll
        for (uint32_t w = 0; w < kWords; ++w) {
            uint64_t v = 0;
#pragma unroll
            for (uint32_t b = 0; b < 8; b += kPiece) {
                const uint32_t idx = 8 * w + b;
                if (idx < sizeof(T)) {
                    if constexpr (kPiece == 4) {
                        uint32_t piece;
                        memcpy(&piece, base + idx, 4);
                        v |= static_cast<uint64_t>(piece) << (8 * b);
                    } else {
                        uint8_t piece;
                        memcpy(&piece, base + idx, 1);
                        v |= static_cast<uint64_t>(piece) << (8 * b);
                    }
                }
            }
            out = (w == i) ? v : out;
        }
        return out;
    }
}

KIWI_DEV uint64_t load_word(const void* p, uint32_t i) {
    return reinterpret_cast<const uint64_t*>(p)[i];
}

}  // namespace dev
#endif  // __CUDACC__

// ---------------------------------------------------------------------------
// Device -> host, single producer warp.
// ---------------------------------------------------------------------------
struct SpscD2HHandle {
    Chunk* ring;                  // device-visible address of the ring
    const uint64_t* consumer_pos; // host-published consumer position (lines)
    ErrorRecord* err;
    uint64_t head;                // producer position (lines), kept in registers
    uint64_t credit_limit;        // head may grow up to this without a PCIe read
    uint32_t log2cap;
    uint32_t pad_;

#if defined(__CUDACC__)
    KIWI_DEV uint64_t capacity() const { return uint64_t{1} << log2cap; }

    /// Credit check; re-reads the consumer position over PCIe (lane 0) only
    /// when the cached credit is short.
    KIWI_DEV bool reserve(uint32_t nlines) {
        if (head + nlines <= credit_limit) return true;
        uint64_t pos = 0;
        if (ptx::lane_id() == 0) pos = ptx::ld_volatile_u64(consumer_pos);
        pos = ptx::bcast64(pos);
        credit_limit = pos + capacity();
        return head + nlines <= credit_limit;
    }

    KIWI_DEV bool oversize(uint32_t bytes) {
        if (bytes <= kMaxMessageBytes && message_lines(bytes) <= capacity()) return false;
        dev::report(err, Status::kOversize, site_d2h_push, bytes);
        return true;
    }

    /// Lane i passes payload word i (bytes <= 256).  Returns false, writing
    /// nothing, if the ring is full.
    KIWI_DEV bool push_lanes(uint64_t word, uint32_t bytes, uint32_t metadata) {
        if (bytes > 32 * 8 || oversize(bytes)) {
            if (bytes > 32 * 8) dev::report(err, Status::kOversize, site_d2h_push, bytes);
            return true;
        }
        const uint32_t nlines = message_lines(bytes);
        if (!reserve(nlines)) return false;
        // Lane l writes chunk l (word l-1) and, for l == 0, chunk 32 (word 31).
        const uint64_t w = ptx::bcast64(word, (ptx::lane_id() + 31) & 31);
        dev::write_message(ring, log2cap, head, bytes, metadata, [&](uint32_t) { return w; });
        head += nlines;
        return true;
    }

    /// The message is a register-resident object every lane holds.
    template <typename T>
    KIWI_DEV bool push_reg(const T& msg, uint32_t metadata = 0) {
        return push_reg_n(msg, sizeof(T), metadata);
    }

    /// As push_reg, sending only the first `bytes` (<= sizeof(T)) bytes of msg.
    template <typename T>
    KIWI_DEV bool push_reg_n(const T& msg, uint32_t bytes, uint32_t metadata = 0) {
        static_assert(sizeof(T) <= 512, "push_reg holds at most 512 bytes in registers");
        if (bytes > sizeof(T)) bytes = sizeof(T);
        if (oversize(bytes)) return true;
        const uint32_t nlines = message_lines(bytes);
        if (!reserve(nlines)) return false;
        dev::write_message(ring, log2cap, head, bytes, metadata,
                           [&](uint32_t i) { return dev::select_word(msg, i); });
        head += nlines;
        return true;
    }

    /// Payload in global memory, 8-byte aligned, readable for round_up(bytes, 8).
    KIWI_DEV bool push_global(const void* ptr, uint32_t bytes, uint32_t metadata = 0) {
        if (oversize(bytes)) return true;
        const uint32_t nlines = message_lines(bytes);
        if (!reserve(nlines)) return false;
        dev::write_message(ring, log2cap, head, bytes, metadata,
                           [&](uint32_t i) { return dev::load_word(ptr, i); });
        head += nlines;
        return true;
    }

    /// Payload in shared memory, 8-byte aligned, published by the caller.
    KIWI_DEV bool push_shared(const void* smem, uint32_t bytes, uint32_t metadata = 0) {
        return push_global(smem, bytes, metadata);  // generic addressing covers shared
    }

    /// One message per active lane, each with its own payload, length and
    /// metadata; consecutive lines in lane order.  All-or-nothing.
    template <typename T>
    KIWI_DEV bool push_lane_masked(const T& msg, uint32_t bytes, uint32_t metadata, bool active) {
        uint32_t my_bytes = active ? bytes : 0;
        bool bad = active && (bytes > sizeof(T) || bytes > kMaxMessageBytes);
        if (__any_sync(ptx::kFullMask, bad)) {
            dev::report(err, Status::kOversize, site_d2h_push, bytes);
            return true;
        }
        const uint32_t my_lines = active ? message_lines(my_bytes) : 0;
        uint32_t total = 0;
        const uint32_t offset = ptx::warp_exclusive_scan(my_lines, total);
        if (total == 0) return true;
        if (total > capacity()) {
            dev::report(err, Status::kOversize, site_d2h_push, total);
            return true;
        }
        if (!reserve(total)) return false;
        if (active) write_own_message(head + offset, msg, my_bytes, metadata);
        head += total;
        return true;
    }

    template <typename T>
    KIWI_DEV void write_own_message(uint64_t at, const T& msg, uint32_t bytes, uint32_t metadata) {
        const uint32_t nchunks = message_chunks(bytes);
        const uint32_t total = message_lines(bytes) * kChunksPerLine;
        const uint64_t mask = capacity() - 1;
        for (uint32_t k = 0; k < total; ++k) {
            const uint64_t line = at + k / kChunksPerLine;
            const uint32_t tag = lap_tag(line, log2cap);
            uint32_t lo = 0, hi = 0;
            if (k == 0) {
                lo = metadata;
                hi = bytes;
            } else if (k < nchunks) {
                const uint64_t w = dev::select_word(msg, k - 1);
                lo = static_cast<uint32_t>(w);
                hi = static_cast<uint32_t>(w >> 32);
            }
            dev::store_chunk(&ring[(line & mask) * kChunksPerLine + (k & 3u)], lo, hi, tag);
        }
    }
#endif
};

// ---------------------------------------------------------------------------
// Device -> host, many producer warps.  Lines are claimed with one
// device-memory atomicAdd per push; a push then waits (bounded) for credit.
// ---------------------------------------------------------------------------
struct MpscD2HHandle {
    Chunk* ring;
    const uint64_t* consumer_pos;
    ErrorRecord* err;
    unsigned long long* claim;    // device-memory producer counter (lines)
    uint64_t credit_limit;        // per-handle credit cache
    uint64_t timeout_ns;
    uint32_t log2cap;
    uint32_t pad_;

#if defined(__CUDACC__)
    KIWI_DEV uint64_t capacity() const { return uint64_t{1} << log2cap; }

    KIWI_DEV bool oversize(uint32_t bytes) {
        if (bytes <= kMaxMessageBytes && message_lines(bytes) <= capacity()) return false;
        dev::report(err, Status::kOversize, site_d2h_push, bytes);
        return true;
    }

    /// Claims `nlines` lines and waits until the consumer has freed them.
    /// Returns false only if the wait timed out (recorded in the ErrorRecord).
    KIWI_DEV bool claim_lines(uint32_t nlines, uint64_t& base) {
        uint64_t b = 0;
        if (ptx::lane_id() == 0) b = atomicAdd(claim, static_cast<unsigned long long>(nlines));
        base = ptx::bcast64(b);
        if (base + nlines <= credit_limit) return true;
        ptx::Deadline dl(timeout_ns);
        uint32_t backoff = 32;
        while (true) {
            uint64_t pos = 0;
            if (ptx::lane_id() == 0) pos = ptx::ld_volatile_u64(consumer_pos);
            pos = ptx::bcast64(pos);
            credit_limit = pos + capacity();
            if (base + nlines <= credit_limit) return true;
            if (dl.expired()) {
                dev::report(err, Status::kTimeout, site_d2h_mpsc_credit, static_cast<uint32_t>(base));
                return false;
            }
            __nanosleep(backoff);
            if (backoff < 1024) backoff <<= 1;
        }
    }

    KIWI_DEV bool push_lanes(uint64_t word, uint32_t bytes, uint32_t metadata) {
        if (bytes > 256) {
            dev::report(err, Status::kOversize, site_d2h_push, bytes);
            return true;
        }
        if (oversize(bytes)) return true;
        uint64_t base;
        if (!claim_lines(message_lines(bytes), base)) return false;
        const uint64_t w = ptx::bcast64(word, (ptx::lane_id() + 31) & 31);
        dev::write_message(ring, log2cap, base, bytes, metadata, [&](uint32_t) { return w; });
        return true;
    }

    template <typename T>
    KIWI_DEV bool push_reg(const T& msg, uint32_t metadata = 0) {
        return push_reg_n(msg, sizeof(T), metadata);
    }

    template <typename T>
    KIWI_DEV bool push_reg_n(const T& msg, uint32_t bytes, uint32_t metadata = 0) {
        static_assert(sizeof(T) <= 512, "push_reg holds at most 512 bytes in registers");
        if (bytes > sizeof(T)) bytes = sizeof(T);
        if (oversize(bytes)) return true;
        uint64_t base;
        if (!claim_lines(message_lines(bytes), base)) return false;
        dev::write_message(ring, log2cap, base, bytes, metadata,
                           [&](uint32_t i) { return dev::select_word(msg, i); });
        return true;
    }

    KIWI_DEV bool push_global(const void* ptr, uint32_t bytes, uint32_t metadata = 0) {
        if (oversize(bytes)) return true;
        uint64_t base;
        if (!claim_lines(message_lines(bytes), base)) return false;
        dev::write_message(ring, log2cap, base, bytes, metadata,
                           [&](uint32_t i) { return dev::load_word(ptr, i); });
        return true;
    }

    KIWI_DEV bool push_shared(const void* smem, uint32_t bytes, uint32_t metadata = 0) {
        return push_global(smem, bytes, metadata);
    }

    template <typename T>
    KIWI_DEV bool push_lane_masked(const T& msg, uint32_t bytes, uint32_t metadata, bool active) {
        const bool bad = active && (bytes > sizeof(T) || bytes > kMaxMessageBytes);
        if (__any_sync(ptx::kFullMask, bad)) {
            dev::report(err, Status::kOversize, site_d2h_push, bytes);
            return true;
        }
        const uint32_t my_lines = active ? message_lines(bytes) : 0;
        uint32_t total = 0;
        const uint32_t offset = ptx::warp_exclusive_scan(my_lines, total);
        if (total == 0) return true;
        if (total > capacity()) {
            dev::report(err, Status::kOversize, site_d2h_push, total);
            return true;
        }
        uint64_t base;
        if (!claim_lines(total, base)) return false;
        if (active) {
            SpscD2HHandle w{ring, consumer_pos, err, 0, 0, log2cap, 0};
            w.write_own_message(base + offset, msg, bytes, metadata);
        }
        return true;
    }
#endif
};

// ---------------------------------------------------------------------------
// Host -> device, single consumer warp.  The host writes messages in the same
// wire format; the warp polls the line at its position with 16-byte volatile
// loads (one 64-byte PCIe read for a one-line message).
// ---------------------------------------------------------------------------
struct SpscH2DHandle {
    const Chunk* ring;
    uint64_t* consumer_pos;       // host memory, written by the consumer (posted)
    ErrorRecord* err;
    uint64_t tail;
    uint64_t published;
    uint32_t log2cap;
    uint32_t notify_interval;     // publish the position after this many lines

#if defined(__CUDACC__)
    KIWI_DEV uint64_t capacity() const { return uint64_t{1} << log2cap; }

    KIWI_DEV const Chunk* chunk_ptr(uint64_t line, uint32_t c) const {
        return &ring[(line & (capacity() - 1)) * kChunksPerLine + c];
    }

    KIWI_DEV void advance(uint32_t nlines) {
        tail += nlines;
        if (tail - published >= notify_interval) flush_consumer_index();
    }

    /// Publishes the consumer position to the host (call before the kernel
    /// exits if notify_interval > 1).
    KIWI_DEV void flush_consumer_index() {
        if (ptx::lane_id() == 0) ptx::st_volatile_u64(consumer_pos, tail);
        published = tail;
    }

    /// Reads and validates the header line.  Returns false if not visible yet.
    KIWI_DEV bool peek_header(uint4& v, uint32_t& bytes, uint32_t& metadata) {
        const uint32_t lane = ptx::lane_id();
        const uint32_t tag = lap_tag(tail, log2cap);
        bool ok = true;
        v = make_uint4(0, 0, 0, 0);
        if (lane < kChunksPerLine) {
            v = ptx::ld_volatile_v4(chunk_ptr(tail, lane));
            ok = dev::chunk_ok(v, tag);
        }
        if (!__all_sync(ptx::kFullMask, ok)) return false;
        metadata = __shfl_sync(ptx::kFullMask, dev::chunk_lo(v), 0);
        bytes = __shfl_sync(ptx::kFullMask, dev::chunk_hi(v), 0);
        if (bytes > kMaxMessageBytes || message_lines(bytes) > capacity()) {
            dev::report(err, Status::kCorrupt, site_h2d_pop, bytes);
            return false;
        }
        return true;
    }

    /// Pops one message of at most 248 bytes into registers: lane i receives
    /// payload word i.  Returns false if no whole message is visible.
    KIWI_DEV bool try_pop(uint64_t& word, uint32_t& bytes, uint32_t& metadata) {
        uint4 v;
        uint32_t len, meta;
        if (!peek_header(v, len, meta)) return false;
        const uint32_t lane = ptx::lane_id();
        const uint32_t nlines = message_lines(len);
        if (len > 31 * 8) {
            dev::report(err, Status::kOversize, site_h2d_pop, len);
            return false;
        }
        if (nlines > 1) {
            const uint32_t total = nlines * kChunksPerLine;
            bool ok = true;
            if (lane < total) {
                const uint64_t line = tail + lane / kChunksPerLine;
                const uint32_t tag = lap_tag(line, log2cap);
                v = ptx::ld_volatile_v4(chunk_ptr(line, lane & 3u));
                ok = dev::chunk_ok(v, tag);
            }
            if (!__all_sync(ptx::kFullMask, ok)) return false;
        }
        // Lane i takes chunk i + 1.
        const uint32_t src = (lane + 1) & 31u;
        const uint32_t lo = __shfl_sync(ptx::kFullMask, dev::chunk_lo(v), src);
        const uint32_t hi = __shfl_sync(ptx::kFullMask, dev::chunk_hi(v), src);
        word = (static_cast<uint64_t>(hi) << 32) | lo;
        bytes = len;
        metadata = meta;
        advance(nlines);
        return true;
    }

    /// Pops one message of any length into `dst` (global or shared memory,
    /// 8-byte aligned, room for round_up(bytes, 8) bytes).
    KIWI_DEV bool try_pop_to(void* dst, uint32_t& bytes, uint32_t& metadata) {
        uint4 v;
        uint32_t len, meta;
        if (!peek_header(v, len, meta)) return false;
        const uint32_t lane = ptx::lane_id();
        const uint32_t nchunks = message_chunks(len);
        const uint32_t total = message_lines(len) * kChunksPerLine;
        uint64_t* out = static_cast<uint64_t*>(dst);
        for (uint32_t base = 0; base < total; base += kWarpSize) {
            const uint32_t k = base + lane;
            bool ok = true;
            if (k < total) {
                const uint64_t line = tail + k / kChunksPerLine;
                const uint32_t tag = lap_tag(line, log2cap);
                const uint4 c = ptx::ld_volatile_v4(chunk_ptr(line, k & 3u));
                ok = dev::chunk_ok(c, tag);
                if (ok && k >= 1 && k < nchunks) {
                    out[k - 1] = (static_cast<uint64_t>(dev::chunk_hi(c)) << 32) | dev::chunk_lo(c);
                }
            }
            if (!__all_sync(ptx::kFullMask, ok)) return false;
        }
        bytes = len;
        metadata = meta;
        advance(message_lines(len));
        return true;
    }

    /// Bounded blocking pop into registers.
    KIWI_DEV Status pop(uint64_t& word, uint32_t& bytes, uint32_t& metadata,
                        uint64_t timeout_ns = kDefaultTimeoutNs) {
        ptx::Deadline dl(timeout_ns);
        while (!try_pop(word, bytes, metadata)) {
            if (dl.expired()) {
                dev::report(err, Status::kTimeout, site_h2d_pop, static_cast<uint32_t>(tail));
                return Status::kTimeout;
            }
        }
        return Status::kOk;
    }
#endif
};

// ---------------------------------------------------------------------------
// Host -> device, many producers (host threads), many consumer warps.  Fixed
// slots of `slot_lines` lines; a consumer claims a slot only after seeing it
// full (CAS on a device counter), then acknowledges it in a per-slot word in
// host memory that producers read locally (Vyukov-style turn per slot).
// ---------------------------------------------------------------------------
struct MpmcH2DHandle {
    const Chunk* ring;
    unsigned long long* claim;    // device-memory consumer counter (slots)
    uint32_t* acks;               // host memory: acks[s] = laps consumed of slot s
    ErrorRecord* err;
    uint32_t log2slots;
    uint32_t slot_lines;

#if defined(__CUDACC__)
    KIWI_DEV uint32_t slot_payload() const { return (slot_lines * kChunksPerLine - 1) * 8; }

    /// Tries to pop one message (at most slot_payload() <= 248 bytes); lane i
    /// receives payload word i.  Returns false if the next slot is empty or
    /// another warp took it first.
    KIWI_DEV bool try_pop(uint64_t& word, uint32_t& bytes, uint32_t& metadata) {
        const uint32_t lane = ptx::lane_id();
        uint64_t pos = 0;
        if (lane == 0) pos = ptx::ld_volatile_u64(claim);
        pos = ptx::bcast64(pos);
        const uint64_t slot = pos & ((uint64_t{1} << log2slots) - 1);
        const uint32_t lap = static_cast<uint32_t>(pos >> log2slots);
        const uint32_t tag = wire_tag(lap);
        const uint32_t total = slot_lines * kChunksPerLine;
        uint4 v = make_uint4(0, 0, 0, 0);
        bool ok = true;
        if (lane < total) {
            v = ptx::ld_volatile_v4(&ring[slot * total + lane]);
            ok = dev::chunk_ok(v, tag);
        }
        if (!__all_sync(ptx::kFullMask, ok)) return false;
        unsigned long long old = 0;
        if (lane == 0) old = atomicCAS(claim, static_cast<unsigned long long>(pos), pos + 1);
        old = ptx::bcast64(old);
        if (old != pos) return false;
        const uint32_t len = __shfl_sync(ptx::kFullMask, dev::chunk_hi(v), 0);
        metadata = __shfl_sync(ptx::kFullMask, dev::chunk_lo(v), 0);
        const uint32_t src = (lane + 1) & 31u;
        const uint32_t lo = __shfl_sync(ptx::kFullMask, dev::chunk_lo(v), src);
        const uint32_t hi = __shfl_sync(ptx::kFullMask, dev::chunk_hi(v), src);
        word = (static_cast<uint64_t>(hi) << 32) | lo;
        bytes = len <= slot_payload() ? len : slot_payload();
        if (len > slot_payload()) dev::report(err, Status::kCorrupt, site_mpmc_pop, len);
        if (lane == 0) ptx::st_volatile_u32(&acks[slot], lap + 1);
        return true;
    }

    KIWI_DEV Status pop(uint64_t& word, uint32_t& bytes, uint32_t& metadata,
                        uint64_t timeout_ns = kDefaultTimeoutNs) {
        ptx::Deadline dl(timeout_ns);
        uint32_t backoff = 0;
        while (!try_pop(word, bytes, metadata)) {
            if (dl.expired()) {
                dev::report(err, Status::kTimeout, site_mpmc_pop, 0);
                return Status::kTimeout;
            }
            if (backoff) __nanosleep(backoff);
            backoff = backoff ? (backoff < 512 ? backoff * 2 : 512) : 16;
        }
        return Status::kOk;
    }
#endif
};

}  // namespace kiwi::queue
