// Host side of kiwi::ep phase timing: phase and meta names, word decoding.
#include "kiwi/ep/debug_timing.hpp"

namespace kiwi::ep {

namespace {
constexpr const char* kPhaseNames[kNumDebugPhases] = {
    "route",        "begin",     "dispatch",     "recv_count",    "recv_assign",  "recv_copy",    "gemm1",
    "gemm2",        "combine_send", "combine_recv", "recv_compact", "gather_rows", "combine_rows",
    "dispatch_wait", "combine_wait",
};
constexpr const char* kMetaNames[kNumDebugMeta] = {
    "rank",          "world",          "tokens",           "recv_tokens",      "recv_remote_tokens",
    "recv_self_tokens", "expert_rows", "dispatch_blocks",  "recv_blocks",      "combine_blocks",
    "hidden",        "topk",           "experts_per_rank", "quant",            "fused_combine",
    "gather_a",      "gemm_pair",
};
}  // namespace

const char* debug_phase_name(int phase) {
    return phase >= 0 && phase < kNumDebugPhases ? kPhaseNames[phase] : nullptr;
}

const char* debug_meta_name(int meta) { return meta >= 0 && meta < kNumDebugMeta ? kMetaNames[meta] : nullptr; }

void decode_debug_words(const uint64_t* raw, uint64_t* out, int n) {
    for (int i = 0; i < n; ++i) {
        const bool start_slot = (i % kDebugWordsPerPhase) % 2 == 0;  // words 0 and 2 of a phase hold ~t
        out[i] = raw[i] == 0 ? 0 : (start_slot ? ~raw[i] : raw[i]);
    }
}

}  // namespace kiwi::ep
