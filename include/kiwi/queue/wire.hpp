// kiwi::queue wire format, shared by every ring in both directions.
//
// Behaviour parity: the reference's device-to-host "LL8" ring
// (include/kiwi/queue/detail/chunk.hip.hpp:1-60 of AMDResearch/kiwi) guards
// every 4 data bytes with a 4-byte signal so that only aligned 8-byte
// single-copy atomicity of PCIe writes and host loads is assumed (the property
// NCCL's LL protocol relies on too).  This file keeps that property and
// defines its own layout:
//
//   ring  = `capacity` 64-byte lines (capacity a power of two)
//   line  = 4 chunks of 16 bytes
//   chunk = { data_lo u32, tag u32, data_hi u32, tag u32 }
//
//   * Every tag is the 32-bit lap tag of the chunk's line:
//         lap_tag(line) = (line >> log2(capacity)) + 1
//     A freshly allocated ring is all zeros (tag 0 = never written), so no
//     initialisation pass is needed, and a full 32-bit compare tells a line of
//     this lap from any earlier lap (not only the previous one).
//   * The message header is in-band: chunk 0's data is {metadata, length}.
//     Payload byte b lives in chunk 1 + b/8.
//   * A message of B bytes occupies message_lines(B) whole lines starting on a
//     line; padding chunks of its last line carry tags (and zero data) so the
//     producer always writes whole 64-byte lines (one PCIe write each) and the
//     consumer can validate a line with one compare of its 8 tags.
//   * A message that reaches the end of the ring continues at line 0 with the
//     next lap's tag.
//
// Each 8-byte half {data, tag} is written by one aligned 8-byte (or wider)
// store and read by one aligned 8-byte (or wider) load, so a reader that sees
// the expected tag in a half sees that half's data.
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

struct alignas(16) Chunk {
    uint32_t lo;
    uint32_t tag0;
    uint32_t hi;
    uint32_t tag1;
};
static_assert(sizeof(Chunk) == kChunkBytes, "chunk is 16 bytes");

KIWI_HD constexpr uint32_t message_chunks(uint32_t bytes) {
    return kHeaderChunks + (bytes + kChunkPayloadBytes - 1) / kChunkPayloadBytes;
}

KIWI_HD constexpr uint32_t message_lines(uint32_t bytes) {
    return (message_chunks(bytes) + kChunksPerLine - 1) / kChunksPerLine;
}

inline constexpr uint32_t kMaxMessageLines = message_lines(kMaxMessageBytes);

KIWI_HD constexpr uint32_t lap_tag(uint64_t line, uint32_t log2_capacity) {
    return static_cast<uint32_t>(line >> log2_capacity) + 1u;
}

/// Packs one 8-byte half {data, tag} as the u64 a single store writes.
KIWI_HD constexpr uint64_t pack_half(uint32_t data, uint32_t tag) {
    return static_cast<uint64_t>(data) | (static_cast<uint64_t>(tag) << 32);
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
