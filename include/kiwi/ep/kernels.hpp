// kiwi::ep device workspace and kernel launchers (csrc/ep_kernels.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "kiwi/ep/config.hpp"
#include "kiwi/p2p/heap.hpp"

namespace kiwi::ep {

/// Rank-local device scratch of one EP layer (allocated by the owner).
struct EpWorkspace {
    uint32_t* epoch;          // [1] round counter, bumped by begin()
    uint32_t* done_ctas;      // [4] last-CTA counters (dispatch, combine)
    int32_t* expert_count;    // [experts_per_rank]
    int32_t* cursor;          // [experts_per_rank]
    int32_t* offsets;         // [experts_per_rank + 1]
    int32_t* tiles1;          // [experts_per_rank + 1] tile prefix of GEMM1
    int32_t* tiles2;          // [experts_per_rank + 1] tile prefix of GEMM2
    int32_t* slot_tokens;     // [world] tokens each source sent this round
    int32_t* pair_slot;       // [max_pairs] source slot of each expert row
    float* pair_w;            // [max_pairs] routing weight of each expert row
    int32_t* slot_pos;        // [slots * local_per_token] expert rows of a slot (-1 = none)
    int64_t* pair_dst;        // [max_pairs] (src rank << 48) | combk_off(token, k) of each expert row
    __nv_bfloat16* a;         // [max_pairs, hidden] dequantised expert-major rows
    uint32_t* error;          // [4] {code, site, info, rank}
    uint64_t* debug_time;     // [kDebugTimeWords] phase stamps (null: timing off)
};

/// Error sites recorded in EpWorkspace::error[1].
enum EpSite : uint32_t {
    kSiteDispatchWait = 1,
    kSiteCombineWait = 2,
    kSiteCapacity = 3,
};

void launch_begin(const EpConfig& c, const EpWorkspace& ws, cudaStream_t s);

/// Blocks launch_dispatch runs for `tokens` tokens: `tuned` when positive,
/// else one warp per token capped at 8 blocks per SM.
int dispatch_grid(int tokens, int tuned, int sms);

/// Top-k routing with softmax over the selected logits (logits fp32 [T, E]).
void launch_route(const float* logits, int tokens, int experts, int topk, int32_t* idx, float* w, cudaStream_t s,
                  uint64_t* debug_time = nullptr);

/// Quantises (per cfg.quant) and stores each token's row, scales and metadata
/// into every destination rank's receive slot; the last CTA signals all ranks.
/// On a bf16 op (Quant::kNone), `raw_scales` [tokens, raw_scale_bytes] are the
/// caller's own per-token scales, carried as bytes next to each row.
void launch_dispatch(const EpConfig& c, const p2p::HeapView& h, const __nv_bfloat16* x, const int32_t* idx,
                     const float* w, int tokens, const EpWorkspace& ws, int grid, cudaStream_t s,
                     const void* raw_scales = nullptr, int raw_scale_bytes = 0);

/// Dispatch of rows the caller already quantised (an FP8 or NVFP4 op): each
/// token's row_bytes of `rows` and scale_row_bytes of `scales` (may be null)
/// travel unchanged into the receive slots (the reference's pre-quantised
/// contract); otherwise as launch_dispatch.
void launch_dispatch_raw(const EpConfig& c, const p2p::HeapView& h, const void* rows, const void* scales,
                         int scale_row_bytes, const int32_t* idx, const float* w, int tokens, const EpWorkspace& ws,
                         int grid, cudaStream_t s);

/// One 32-thread block waits (bounded) for every rank's dispatch (which = 0)
/// or combine (which = 1) flag of this round; for dispatch it records each
/// source's token count.  Launch it ahead of the kernel that reads the data
/// and pass waited = true to that kernel: then the only kernel that spins on
/// other GPUs is this one, which cannot keep a kernel of another stream from
/// being scheduled.
void launch_wait_flags(const EpConfig& c, const p2p::HeapView& h, const EpWorkspace& ws, int which,
                       uint64_t timeout_ns, cudaStream_t s);

/// Counts rows per local expert, after waiting for every source's dispatch
/// flag itself (waited = false) or after launch_wait_flags(which = 0).
void launch_recv_count(const EpConfig& c, const p2p::HeapView& h, const EpWorkspace& ws, uint64_t timeout_ns,
                       cudaStream_t s, bool waited = false);

/// Assigns expert-major rows: pair_slot / pair_w / pair_dst of every row and
/// the slot -> rows map (slot_pos).
void launch_recv_assign(const EpConfig& c, const p2p::HeapView& h, const EpWorkspace& ws, cudaStream_t s,
                        int grid = 0);

/// Dequantises each received row into its expert-major rows of ws.a (not
/// needed when GEMM1 gathers its A operand from the receive buffer).
void launch_recv_copy(const EpConfig& c, const p2p::HeapView& h, const EpWorkspace& ws, cudaStream_t s,
                      int grid = 0);

/// launch_recv_assign then launch_recv_copy.
void launch_recv_scatter(const EpConfig& c, const p2p::HeapView& h, const EpWorkspace& ws, cudaStream_t s);

/// Sums each slot's (already weighted) expert outputs y and stores the bf16
/// row into the source rank's combine slot; the last CTA signals all ranks.
void launch_combine_send(const EpConfig& c, const p2p::HeapView& h, const __nv_bfloat16* y, const EpWorkspace& ws,
                         int grid, cudaStream_t s);

/// Waits for every rank's combine flag and reduces the returned rows of each
/// local token (over the ranks it was sent to), in fp32, into out [T,
/// comb_row_bytes] in the op's combine dtype.  With out_w [T, topk] (an op
/// whose comb slots carry weights), each token's returned top-k weights are
/// summed there too.
void launch_combine_recv(const EpConfig& c, const p2p::HeapView& h, const int32_t* idx, int tokens, void* out,
                         const EpWorkspace& ws, uint64_t timeout_ns, cudaStream_t s, int grid = 0,
                         float* out_w = nullptr, bool waited = false);

/// Fused combine, receive side: after every rank's combine flag (set by the
/// last CTA of each rank's scatter GEMM2), sums each local token's top-k rows
/// of combk (already routing-weighted) into out [T, hidden].
void launch_combine_recv_fused(const EpConfig& c, const p2p::HeapView& h, const int32_t* idx, int tokens,
                               __nv_bfloat16* out, const EpWorkspace& ws, uint64_t timeout_ns, cudaStream_t s,
                               int grid = 0, bool waited = false);

// ---- transport-only (MORI-compatible) path ----

/// One block: deterministic compaction of this round's valid slots in
/// (source rank, token) order; slot_compact[s] = output row or -1, *recv_count = total.
/// Call after launch_recv_count (which waited for every source).
void launch_recv_compact(const EpConfig& c, const p2p::HeapView& h, const EpWorkspace& ws, int32_t* slot_compact,
                         int32_t* recv_count, cudaStream_t s);

/// Copies each valid slot's row (wire bytes), scales, top-k ids and weights into
/// the compacted outputs and records src_pos = src * max_tokens + token.
void launch_gather_rows(const EpConfig& c, const p2p::HeapView& h, const EpWorkspace& ws,
                        const int32_t* slot_compact, uint8_t* out_rows, uint8_t* out_scales, int32_t* out_idx,
                        float* out_w, int32_t* out_src_pos, cudaStream_t s);

/// Sends row i of `rows` ([recv_count, comb_row_bytes] in the combine dtype,
/// 16-byte aligned) and, when given, its top-k `weights` (fp32 [recv_count,
/// topk]) to its token's rank (src_pos[i]); the last CTA signals every rank's
/// combine flag.
void launch_combine_rows(const EpConfig& c, const p2p::HeapView& h, const void* rows, const float* weights,
                         const int32_t* src_pos, const int32_t* recv_count, const EpWorkspace& ws, cudaStream_t s);

}  // namespace kiwi::ep
