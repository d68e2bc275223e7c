// kiwi::ep launch tuning for B200.
//
// Parity with the reference's runtime tuning tables (apps/ep/ep_tuning.hpp:18-128
// of AMDResearch/kiwi), which pick block counts and the transport backend per
// (GPU architecture, NIC family) from measured tables with a generic
// fallback.  On B200 every peer is one NVSwitch hop away, so there is no
// transport choice; the table picks the grid of each EP kernel and which
// fused paths the layer uses, keyed by the rank's token capacity, and records
// where each choice was measured.  KIWI_EP_TUNING="key=value,..." overrides
// any field (keys: dispatch_blocks, recv_blocks, combine_blocks,
// fused_combine, gather_a, gemm_pair, gemm_pair_auto, gemm_split, gemm2_pair,
// gemm_m64_tails).
#pragma once

#include <string>

#include "kiwi/ep/config.hpp"

namespace kiwi::ep {

struct EpTuning {
    int32_t dispatch_blocks;  // 0: one warp per token, at most 8 blocks per SM
    int32_t recv_blocks;      // receive copy / assign grid
    int32_t combine_blocks;   // combine send / reduce grid
    bool fused_combine;       // GEMM2 epilogue stores over NVLink
    bool gather_a;            // GEMM1 gathers A from the receive slots
    bool gemm_pair;           // 2-SM (256-row tile) grouped GEMMs alone in every round
    bool gemm_pair_auto;      // 2-SM GEMMs in rounds expecting kPairMinRows rows per local expert
    bool gemm_split;          // 2-SM pass over full 256-row tiles + 1-SM pass over the tails, every round
    bool gemm_m64_tails;      // 1-SM GEMMs: M = 64 MMAs for tiles with <= 64 rows of their expert left
    bool gemm2_pair;          // down projection (GEMM2) on the 2-SM kernel, gate/up (GEMM1) on the 1-SM one;
                              // one B200 at 1024 rows per expert: 25.09 vs 23.19 ms per step (1-SM both)
    std::string source;       // table entry (and overrides) this came from
};

/// Expected rows per local expert from which a round runs the 2-SM GEMMs
/// (256-row tiles).  Under the B200's power cap the 2-SM kernels lost where an
/// expert's last, part-padding tile is a noticeable share of its rows: at 8
/// GPUs 3.09 vs 2.90 ms per step with 1024 rows per expert, and on one GPU with
/// 1024 rows per expert the split variant (2-SM over full tiles, 1-SM over the
/// tails) took 27.0 vs 22.5 ms at a median clock of 1102 vs 1387 MHz; with 6144
/// rows per expert (the NVFP4 config at 8 GPUs) they won, 3.22 vs 3.36 ms.
inline constexpr int kPairMinRows = 4096;

/// Tuning for configuration `c` on a GPU with `sms` SMs, then the
/// KIWI_EP_TUNING overrides (`env` stands in for the variable in tests;
/// nullptr reads the process environment).  Throws kiwi::error on a bad
/// override string.
EpTuning tune(const EpConfig& c, int sms, const char* env = nullptr);

}  // namespace kiwi::ep
