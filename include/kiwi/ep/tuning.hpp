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
// fused_combine, gather_a, gemm_pair, gemm_pair_auto).
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
    bool gemm_pair;           // 2-SM (256-row tile) grouped GEMMs in every round
    bool gemm_pair_auto;      // 2-SM GEMMs in rounds whose expected rows per local expert reach kPairMinRows
    std::string source;       // table entry (and overrides) this came from
};

/// Expected rows per local expert from which a round uses the 2-SM GEMMs.
/// The last tile of every expert is part padding (on average half a tile: 128
/// rows with 256-row tiles, 64 with 128-row ones), which has to be small
/// against the 2-SM kernel's gain: measured at 8 B200s, 1024 rows per expert
/// (the FP8 headline config) ran 6.6 % slower with the 2-SM GEMMs and 6144
/// rows (the NVFP4 config) 4 % faster.
inline constexpr int kPairMinRows = 2048;

/// Tuning for configuration `c` on a GPU with `sms` SMs, then the
/// KIWI_EP_TUNING overrides (`env` stands in for the variable in tests;
/// nullptr reads the process environment).  Throws kiwi::error on a bad
/// override string.
EpTuning tune(const EpConfig& c, int sms, const char* env = nullptr);

}  // namespace kiwi::ep
