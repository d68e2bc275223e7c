// kiwi::queue wire format, shared by every ring in both directions.
//
// Behaviour parity: the reference's device-to-host "LL8" ring
// (include/kiwi/queue/detail/chunk.hip.hpp:1-60 of AMDResearch/kiwi) guards
// every 4 data bytes with a 4-byte signal and assumes that an aligned 8-byte
// PCIe write is seen whole by a host 8-byte load.  On the B200 hosts this was
// built on that assumption does NOT hold: a host hammering one line that a
// kernel rewrote with 16- or 8-byte stores saw ~1 in 1000 reads with the high
// 4 bytes of an 8-byte word newer than the low 4 bytes (the atomicity test in
// the bench module reproduces it).  Single 4-byte words were never torn.  So
// this layout puts a tag in EVERY 32-bit word:
//
//   ring  = `capacity` 64-byte lines (capacity a power of two)
//   line  = 4 chunks of 16 bytes
//   chunk = 4 tagged words; word j = { data bits [16j, 16j+16) : 16, tag : 16 }
//           (data in the low half of the word, the tag in the high half), so a
//           chunk carries 8 payload bytes, the same 50% as data+tag halves.
//
//   * A tag is the 16-bit wire tag of the chunk's lap:
//         lap_tag(line) = wire_tag(line >> log2(capacity))
//         wire_tag(n)   = n % 65535 + 1            (1 .. 65535, never 0)
//     A freshly allocated ring is all zeros (tag 0 = never written), so no
//     initialisation pass is needed.  The producer is never more than one lap
//     ahead of the consumer (credit), so the only stale tag a reader can meet
//     is the previous lap's, which differs from the expected one.
//   * The message header is in-band: chunk 0's data is {metadata, length}.
//     Payload byte b lives in chunk 1 + b/8.
//   * A message of B bytes occupies message_lines(B) whole lines starting on a
//     line; padding chunks of its last line carry tags (and zero data) so the
//     producer always writes whole 64-byte lines (one PCIe write each).  The
//     consumer validates every chunk of the message's lines, padding included
//     (one masked compare of a chunk's 4 tags), before it advances and grants
//     the lines back as credit.
//   * A message that reaches the end of the ring continues at line 0 with the
//     next lap's tag.
//
// Measured on B200 hosts (the atomicity tests of the bench module): while a
// kernel rewrote one line back to back, host 8-byte loads sometimes returned
// ZERO for a half (never a mix of the old and new values), and a host reading
// a line that a kernel writes once per round (the ring pattern) saw only the
// old or the new value.  So the format assumes that a 4-byte word being
// rewritten reads as its old value, its new value or zero; since no tag is 0,
// a reader that sees the expected tag in a word sees that word's data.
#pragma once

#include "kiwi/common.hpp"

namespace kiwi::queue {

inline constexpr uint32_t kChunkBytes = 16;
inline constexpr uint32_t kLineBytes = 64;
inline constexpr uint32_t kChunksPerLine = 4;
inline constexpr uint32_t kChunkPayloadBytes = 8;
inline constexpr uint32_t kHeaderChunks = 1;
/// Largest message.  4 KB covers the invoke payload sweep (8 B - 4 KB); a
/// 32-lane warp writes it with 17 stores per lane.
inline constexpr uint32_t kMaxMessageBytes = 4096;
/// Largest ring, in lines: in-flight line counts stay below 2^31.
inline constexpr uint64_t kMaxCapacityLines = uint64_t{1} << 31;
/// Width of the warp that runs every collective device operation on B200.
inline constexpr uint32_t kWarpSize = 32;

/// One 16-byte chunk as two 8-byte halves; each half is two tagged words
/// carrying 32 data bits (see pack_half).
struct alignas(16) Chunk {
    uint64_t lo;
    uint64_t hi;
};
static_assert(sizeof(Chunk) == kChunkBytes, "chunk is 16 bytes");

KIWI_HD constexpr uint32_t message_chunks(uint32_t bytes) {
    return kHeaderChunks + (bytes + kChunkPayloadBytes - 1) / kChunkPayloadBytes;
}

KIWI_HD constexpr uint32_t message_lines(uint32_t bytes) {
    return (message_chunks(bytes) + kChunksPerLine - 1) / kChunksPerLine;
}

inline constexpr uint32_t kMaxMessageLines = message_lines(kMaxMessageBytes);

/// 16-bit tag of round `n` (a lap or a reply sequence number): 1 .. 65535,
/// so consecutive rounds differ and a zeroed word never matches.
KIWI_HD constexpr uint32_t wire_tag(uint64_t n) { return static_cast<uint32_t>(n % 65535u) + 1u; }

KIWI_HD constexpr uint32_t lap_tag(uint64_t line, uint32_t log2_capacity) {
    return wire_tag(line >> log2_capacity);
}

/// One tagged word: 16 data bits (the low half of `data16`) and the low 16
/// bits of `tag` in the high half.
KIWI_HD constexpr uint32_t tagged_word(uint32_t data16, uint32_t tag) {
    return (data16 & 0xffffu) | (tag << 16);
}

/// True if every word among a..d carries `tag` (one masked compare).
KIWI_HD constexpr bool words_have_tag(uint32_t a, uint32_t b, uint32_t c, uint32_t d, uint32_t tag) {
    const uint32_t t = tag << 16;
    return (((a ^ t) | (b ^ t) | (c ^ t) | (d ^ t)) >> 16) == 0;
}

/// The 32 data bits of two tagged words (w0 holds the low 16).
KIWI_HD constexpr uint32_t join_words(uint32_t w0, uint32_t w1) { return (w0 & 0xffffu) | (w1 << 16); }

/// Packs 32 data bits as one 8-byte half: two tagged words.
KIWI_HD constexpr uint64_t pack_half(uint32_t data, uint32_t tag) {
    return static_cast<uint64_t>(tagged_word(data, tag)) |
           (static_cast<uint64_t>(tagged_word(data >> 16, tag)) << 32);
}

/// True if both words of half `h` carry `tag`.
KIWI_HD constexpr bool half_has_tag(uint64_t h, uint32_t tag) {
    const uint64_t t = tag & 0xffffu;
    return (h & 0xffff0000ffff0000ull) == ((t << 16) | (t << 48));
}

/// The 32 data bits of half `h`.
KIWI_HD constexpr uint32_t half_data(uint64_t h) {
    return join_words(static_cast<uint32_t>(h), static_cast<uint32_t>(h >> 32));
}

/// Host-side queue configuration check shared by every ring constructor.
inline void check_capacity(uint64_t capacity_lines) {
    if (!is_pow2(capacity_lines)) {
        throw kiwi::error("kiwi::queue capacity must be a non-zero power of two, got " +
                          std::to_string(capacity_lines));
    }
    if (capacity_lines > kMaxCapacityLines) {
        throw kiwi::error("kiwi::queue capacity exceeds kMaxCapacityLines (2^31)");
    }
}

}  // namespace kiwi::queue
