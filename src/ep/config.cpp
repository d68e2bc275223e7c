#include "kiwi/ep/config.hpp"

#include <string>

namespace kiwi::ep {

EpConfig finalize(EpConfig c) {
    auto bad = [](const std::string& m) { throw kiwi::error("kiwi::ep config: " + m); };
    if (c.world < 1 || c.world > kMaxRanks) bad("world must be in [1, 16]");
    if (c.rank < 0 || c.rank >= c.world) bad("rank out of range");
    if (c.num_experts < 1 || c.num_experts % c.world != 0) bad("num_experts must be a positive multiple of world");
    c.experts_per_rank = c.num_experts / c.world;
    if (c.topk < 1 || c.topk > kMaxTopk || c.topk > c.num_experts) bad("topk must be in [1, min(16, num_experts)]");
    if (c.max_tokens < 1) bad("max_tokens must be positive");
    if (c.hidden < 1) bad("hidden must be positive");
    switch (static_cast<Quant>(c.quant)) {
        case Quant::kNone:
            if (c.hidden % 8 != 0) bad("bf16 dispatch needs hidden % 8 == 0");
            c.row_bytes = c.hidden * 2;
            c.scale_bytes = 0;
            break;
        case Quant::kFp8:
            if (c.hidden % 512 != 0) bad("FP8 dispatch needs hidden % 512 == 0");
            c.row_bytes = c.hidden;
            c.scale_bytes = static_cast<int32_t>(round_up(static_cast<uint64_t>(c.hidden / kFp8Block) * 4, 16));
            break;
        case Quant::kNvfp4:
            if (c.hidden % 512 != 0) bad("NVFP4 dispatch needs hidden % 512 == 0");
            c.row_bytes = c.hidden / 2;
            // e4m3 scale per 16 elements + one fp32 row scale, padded to 16 bytes.
            c.scale_bytes = static_cast<int32_t>(round_up(static_cast<uint64_t>(c.hidden / kFp4Block) + 4, 16));
            break;
        default:
            bad("unknown quant format");
    }
    if (c.min_scale_bytes < 0) bad("min_scale_bytes must be >= 0");
    if (c.min_scale_bytes > c.scale_bytes) c.scale_bytes = static_cast<int32_t>(round_up(c.min_scale_bytes, 16));
    switch (static_cast<CombDtype>(c.comb_dtype)) {
        case CombDtype::kBf16: c.comb_row_bytes = c.hidden * 2; break;
        case CombDtype::kF32: c.comb_row_bytes = c.hidden * 4; break;
        case CombDtype::kFp8: c.comb_row_bytes = c.hidden; break;
        case CombDtype::kFp4:
            if (c.hidden % 2 != 0) bad("FP4 combine needs an even hidden");
            c.comb_row_bytes = c.hidden / 2;
            break;
        default:
            bad("unknown combine dtype");
    }
    if (c.comb_row_bytes % 16 != 0) bad("combine rows must be a multiple of 16 bytes (hidden too small or odd)");
    c.comb_bytes = c.comb_row_bytes + (c.comb_weights ? static_cast<int32_t>(round_up(4ull * c.topk, 16)) : 0);
    c.meta_bytes = static_cast<int32_t>(round_up(sizeof(DispatchMetaHeader) + 8ull * c.topk, 16));
    const uint64_t slots = c.slots();
    uint64_t off = 0;
    c.off_flags = off;
    off += round_up(2 * kMaxRanks * kFlagStride, 256);
    c.off_meta = off;
    off += round_up(slots * c.meta_bytes, 256);
    c.off_row = off;
    off += round_up(slots * c.row_bytes, 256);
    c.off_scale = off;
    off += round_up(slots * static_cast<uint64_t>(c.scale_bytes), 256);
    c.off_comb = off;
    off += round_up(slots * static_cast<uint64_t>(c.comb_bytes), 256);
    c.off_combk = off;
    off += round_up(static_cast<uint64_t>(c.max_tokens) * c.topk * static_cast<uint64_t>(c.hidden) * 2, 256);
    c.heap_bytes = off;
    return c;
}

}  // namespace kiwi::ep
