// kiwi::ep configuration and memory layout (host + device).
//
// Parity: the reference's config_t and heap layout (apps/ep/ep_config.hpp:144-507
// of AMDResearch/kiwi): world size, experts, hidden size, top-k (<= 16),
// per-rank token capacity, quantisation format and the derived slot layout of
// one symmetric heap holding receive slots, combine slots and readiness flags.
// B200 layout (all ranks identical, so a peer address is base[r] + offset):
//
//   flags       dispatch_done[src] and combine_done[src], one u64 per rank,
//               value (epoch << 32) | token_count, 128-byte stride
//   recv_meta   [src][token] DispatchMeta: epoch, top-k ids and weights
//   recv_row    [src][token] the dispatched row (FP8 / NVFP4 / BF16 bytes)
//   recv_scale  [src][token] block scales (FP8: fp32 per 128; NVFP4: e4m3 per 16 + fp32 row scale)
//   comb        [expert_owner][token] rows returned by combine (comb_bytes per
//               slot: the row in comb_dtype, then its top-k fp32 weights when
//               comb_weights is set)
//   combk       [token][k] bf16 rows written by the fused GEMM2 epilogue of
//               the rank that owns the token's k-th expert (routing weight
//               applied), summed over k by the receive side
//
// A slot is valid for a round when its meta.epoch equals the round's epoch,
// so nothing is cleared between rounds.
#pragma once

#include <cstdint>

#include "kiwi/common.hpp"
#include "kiwi/p2p/heap.hpp"

namespace kiwi::ep {

using p2p::kMaxRanks;

enum class Quant : int32_t { kNone = 0, kFp8 = 1, kNvfp4 = 2 };

/// Element type of combine rows: bf16, fp32, FP8 e4m3 codes (no scales) or
/// packed FP4 e2m1 codes (two per byte, element 2i in the low nibble).
enum class CombDtype : int32_t { kBf16 = 0, kF32 = 1, kFp8 = 2, kFp4 = 3 };

inline constexpr int kMaxTopk = 16;
inline constexpr int kFp8Block = 128;   // 1 x 128 block scaling
inline constexpr int kFp4Block = 16;    // NVFP4: 16-element blocks, e4m3 scales
inline constexpr uint64_t kFlagStride = 128;

struct EpConfig {
    int32_t world;
    int32_t rank;
    int32_t hidden;
    int32_t num_experts;
    int32_t experts_per_rank;
    int32_t topk;
    int32_t max_tokens;
    int32_t quant;        // Quant
    int32_t comb_dtype;   // CombDtype of the comb slots (bf16 by default)
    int32_t comb_weights; // 1: comb slots also carry each row's top-k weights
    int32_t min_scale_bytes;  // per-row scale room a caller's own scales need (0: the format's)
    // Derived by finalize():
    int32_t row_bytes;    // dispatched row payload
    int32_t scale_bytes;  // per-row scale bytes (16-byte multiple)
    int32_t meta_bytes;   // DispatchMeta size (16-byte multiple)
    int32_t comb_row_bytes;  // bytes of one combine row in comb_dtype (16-byte multiple)
    int32_t comb_bytes;      // bytes of one comb slot (row + weights, 16-byte multiple)
    uint64_t off_flags;
    uint64_t off_meta;
    uint64_t off_row;
    uint64_t off_scale;
    uint64_t off_comb;
    uint64_t off_combk;
    uint64_t heap_bytes;

    KIWI_HD uint64_t slots() const { return static_cast<uint64_t>(world) * max_tokens; }
    KIWI_HD uint64_t slot_index(int src, int token) const {
        return static_cast<uint64_t>(src) * max_tokens + token;
    }
    KIWI_HD uint64_t dispatch_flag(int src) const { return off_flags + kFlagStride * src; }
    KIWI_HD uint64_t combine_flag(int src) const { return off_flags + kFlagStride * (kMaxRanks + src); }
    KIWI_HD uint64_t meta_off(uint64_t slot) const { return off_meta + slot * meta_bytes; }
    KIWI_HD uint64_t row_off(uint64_t slot) const { return off_row + slot * row_bytes; }
    KIWI_HD uint64_t scale_off(uint64_t slot) const { return off_scale + slot * scale_bytes; }
    KIWI_HD uint64_t comb_off(int owner, int token) const {
        return off_comb + (static_cast<uint64_t>(owner) * max_tokens + token) * static_cast<uint64_t>(comb_bytes);
    }
    KIWI_HD uint64_t combk_off(int token, int k) const {
        return off_combk + (static_cast<uint64_t>(token) * topk + k) * static_cast<uint64_t>(hidden) * 2;
    }
    /// Upper bound of (token, local expert) pairs a rank can receive.
    KIWI_HD int64_t max_pairs() const {
        const int per_token = topk < experts_per_rank ? topk : experts_per_rank;
        return static_cast<int64_t>(world) * max_tokens * per_token;
    }
    KIWI_HD int local_per_token() const { return topk < experts_per_rank ? topk : experts_per_rank; }
};

/// Validates the configuration and fills the derived fields; throws kiwi::error.
EpConfig finalize(EpConfig c);

/// Per-token metadata written with the row (16-byte multiple).
struct alignas(16) DispatchMetaHeader {
    uint32_t epoch;
    uint32_t token;
    uint32_t pad0;
    uint32_t pad1;
    // followed by int32 ids[topk], float weights[topk]
};

}  // namespace kiwi::ep
