// kiwi::ep device phase timing (opt-in).  When enabled, every EP kernel and
// both expert GEMMs stamp %globaltimer (nanoseconds) into a small device buffer;
// the host reads it after the round (get_debug_timing_snapshot).
//
// Parity: the reference's debug_time_buf / debug_time_meta, switched by
// set_debug_timing_enabled and read by get_debug_timing_snapshot
// (AMDResearch/kiwi apps/ep/ep_context.hip.cpp:601-617, apps/ep/dispatch.hip.cpp:32-45
// and :120-134, apps/ep/combine.hip.cpp:105-119 and :607-1030,
// apps/ep/python/kiwi_ep_bindings.hip.cpp:471-506).  The reference stamps
// named points of block 0 into one 64-word buffer that the next kernel
// overwrites.  Here each kernel (phase) owns four words:
//
//   [4p + 0]  first block start   stored as ~t with atomicMax (0 = not recorded)
//   [4p + 1]  last warp end       atomicMax(t)
//   [4p + 2]  block 0's flag wait start   ~t with atomicMax  (kernels that wait on flags)
//   [4p + 3]  block 0's flag wait end     atomicMax(t)
//
// so one round leaves every kernel's span over ALL its blocks side by side,
// and a single zeroing memset at the start of a round resets every slot.
// Disabled (null buffer) the stamps cost one predicated branch per block.
#pragma once

#include <cstdint>

#include "kiwi/common.hpp"
#if defined(__CUDACC__)
#include "kiwi/ptx.cuh"
#endif

namespace kiwi::ep {

enum DebugPhase : int {
    kPhaseRoute = 0,
    kPhaseBegin,
    kPhaseDispatch,
    kPhaseRecvCount,
    kPhaseRecvAssign,
    kPhaseRecvCopy,
    kPhaseGemm1,
    kPhaseGemm2,
    kPhaseCombineSend,
    kPhaseCombineRecv,
    kPhaseRecvCompact,
    kPhaseGatherRows,
    kPhaseCombineRows,
    kPhaseDispatchWait,  // wait_flags_kernel ahead of recv_count
    kPhaseCombineWait,   // wait_flags_kernel ahead of the combine reduce
    kNumDebugPhases
};

inline constexpr int kDebugWordsPerPhase = 4;
inline constexpr int kDebugTimeWords = 64;  // >= kNumDebugPhases * kDebugWordsPerPhase
inline constexpr int kDebugMetaWords = 32;
static_assert(kNumDebugPhases * kDebugWordsPerPhase <= kDebugTimeWords, "debug buffer too small");

/// Name of a phase ("dispatch", "gemm1", ...), nullptr past the end.
const char* debug_phase_name(int phase);

/// Meta words a snapshot fills (host side, from the workspace of the round).
enum DebugMeta : int {
    kMetaRank = 0,
    kMetaWorld,
    kMetaTokens,
    kMetaRecvTokens,
    kMetaRecvRemote,
    kMetaRecvSelf,
    kMetaExpertRows,
    kMetaDispatchBlocks,
    kMetaRecvBlocks,
    kMetaCombineBlocks,
    kMetaHidden,
    kMetaTopk,
    kMetaExpertsPerRank,
    kMetaQuant,
    kMetaFusedCombine,
    kMetaGatherA,
    kMetaGemmPair,  // 0: 1-SM GEMMs, 1: 2-SM both, 2: split (2-SM + 1-SM tails), 3: GEMM2 alone on 2-SM
    kNumDebugMeta
};
static_assert(kNumDebugMeta <= kDebugMetaWords, "meta buffer too small");

const char* debug_meta_name(int meta);

/// Decodes raw device words into absolute nanoseconds (0 = not recorded):
/// start slots hold ~t, end slots hold t.
void decode_debug_words(const uint64_t* raw, uint64_t* out, int n);

#if defined(__CUDACC__)

/// Records one kernel's span: construct first thing in the kernel (every
/// thread); the destructor stamps each warp's exit on every return path.
struct PhaseScope {
    uint64_t* w;

    KIWI_DEV PhaseScope(uint64_t* buf, int phase) : w(buf ? buf + kDebugWordsPerPhase * phase : nullptr) {
        if (w && threadIdx.x == 0) atomicMax(reinterpret_cast<unsigned long long*>(w), ~ptx::globaltimer());
    }
    KIWI_DEV ~PhaseScope() {
        if (w && (threadIdx.x & 31) == 0) atomicMax(reinterpret_cast<unsigned long long*>(w + 1), ptx::globaltimer());
    }
    /// Call from the thread(s) that wait, before and after the wait.  Only
    /// block 0 records: later waves of a multi-wave grid start waiting later,
    /// which would make the span the launch spread rather than the wait.
    KIWI_DEV void wait_begin() const {
        if (w && blockIdx.x == 0) atomicMax(reinterpret_cast<unsigned long long*>(w + 2), ~ptx::globaltimer());
    }
    KIWI_DEV void wait_end() const {
        if (w && blockIdx.x == 0) atomicMax(reinterpret_cast<unsigned long long*>(w + 3), ptx::globaltimer());
    }
    PhaseScope(const PhaseScope&) = delete;
    PhaseScope& operator=(const PhaseScope&) = delete;
};

/// Start and end stamps of a kernel with a structured exit (the GEMMs): one
/// thread per block calls each.
KIWI_DEV void span_start(uint64_t* span) {
    if (span) atomicMax(reinterpret_cast<unsigned long long*>(span), ~ptx::globaltimer());
}
KIWI_DEV void span_end(uint64_t* span) {
    if (span) atomicMax(reinterpret_cast<unsigned long long*>(span + 1), ptx::globaltimer());
}

#endif  // __CUDACC__

}  // namespace kiwi::ep
