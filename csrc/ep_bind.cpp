// Python bindings of kiwi::ep: the fused expert-parallel MoE layer.
//
// Parity: the reference's KiwiEpOp (apps/ep/python/kiwi_ep_bindings.hip.cpp:123-574
// of AMDResearch/kiwi) binds dispatch/combine of rows only.  MoeLayer binds the
// whole B200 layer: routing, FP8/NVFP4 dispatch over NVLink, expert-major
// layout, the two tcgen05 grouped GEMMs (SwiGLU fused into the first, routing
// weight into the second), combine over NVLink and the final reduction, all
// enqueued on the current torch stream with no host synchronisation.
#include <ATen/cuda/CUDAContext.h>
#include <array>
#include <cstring>
#include <vector>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <torch/extension.h>

#include "kiwi/ep/config.hpp"
#include "kiwi/ep/debug_timing.hpp"
#include "kiwi/ep/kernels.hpp"
#include "kiwi/ep/tuning.hpp"
#include "kiwi/gemm/grouped_gemm.hpp"
#include "kiwi/p2p/heap.hpp"

namespace py = pybind11;
using namespace kiwi;

namespace {

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

ep::EpConfig config_from_dict(const py::dict& d) {
    ep::EpConfig c{};
    c.world = d["world"].cast<int>();
    c.rank = d["rank"].cast<int>();
    c.hidden = d["hidden"].cast<int>();
    c.num_experts = d["num_experts"].cast<int>();
    c.topk = d["topk"].cast<int>();
    c.max_tokens = d["max_tokens"].cast<int>();
    if (d.contains("comb_dtype")) {
        if (py::isinstance<py::int_>(d["comb_dtype"])) {
            c.comb_dtype = d["comb_dtype"].cast<int>();
        } else {
            const std::string cd = d["comb_dtype"].cast<std::string>();
            if (cd == "bf16") c.comb_dtype = static_cast<int>(ep::CombDtype::kBf16);
            else if (cd == "f32" || cd == "float32") c.comb_dtype = static_cast<int>(ep::CombDtype::kF32);
            else if (cd == "fp8") c.comb_dtype = static_cast<int>(ep::CombDtype::kFp8);
            else if (cd == "fp4") c.comb_dtype = static_cast<int>(ep::CombDtype::kFp4);
            else throw kiwi::error("unknown combine dtype " + cd);
        }
    }
    if (d.contains("comb_weights")) c.comb_weights = d["comb_weights"].cast<bool>() ? 1 : 0;
    if (d.contains("min_scale_bytes")) c.min_scale_bytes = d["min_scale_bytes"].cast<int>();
    if (py::isinstance<py::int_>(d["quant"])) {
        c.quant = d["quant"].cast<int>();
        return ep::finalize(c);
    }
    const std::string q = d["quant"].cast<std::string>();
    if (q == "none" || q == "bf16") c.quant = static_cast<int>(ep::Quant::kNone);
    else if (q == "fp8") c.quant = static_cast<int>(ep::Quant::kFp8);
    else if (q == "nvfp4" || q == "fp4") c.quant = static_cast<int>(ep::Quant::kNvfp4);
    else throw kiwi::error("unknown quant format " + q);
    return ep::finalize(c);
}

py::dict config_to_dict(const ep::EpConfig& c) {
    py::dict d;
    d["world"] = c.world;
    d["rank"] = c.rank;
    d["hidden"] = c.hidden;
    d["num_experts"] = c.num_experts;
    d["experts_per_rank"] = c.experts_per_rank;
    d["topk"] = c.topk;
    d["max_tokens"] = c.max_tokens;
    d["quant"] = c.quant;
    d["comb_dtype"] = c.comb_dtype;
    d["comb_weights"] = c.comb_weights;
    d["min_scale_bytes"] = c.min_scale_bytes;
    d["comb_row_bytes"] = c.comb_row_bytes;
    d["comb_bytes"] = c.comb_bytes;
    d["row_bytes"] = c.row_bytes;
    d["scale_bytes"] = c.scale_bytes;
    d["meta_bytes"] = c.meta_bytes;
    d["off_flags"] = c.off_flags;
    d["off_meta"] = c.off_meta;
    d["off_row"] = c.off_row;
    d["off_scale"] = c.off_scale;
    d["off_comb"] = c.off_comb;
    d["off_combk"] = c.off_combk;
    d["heap_bytes"] = c.heap_bytes;
    d["max_pairs"] = c.max_pairs();
    d["local_per_token"] = c.local_per_token();
    return d;
}

py::dict tuning_dict(const ep::EpTuning& t) {
    py::dict d;
    d["dispatch_blocks"] = t.dispatch_blocks;
    d["recv_blocks"] = t.recv_blocks;
    d["combine_blocks"] = t.combine_blocks;
    d["fused_combine"] = t.fused_combine;
    d["gather_a"] = t.gather_a;
    d["gemm_pair"] = t.gemm_pair;
    d["gemm_pair_auto"] = t.gemm_pair_auto;
    d["gemm_split"] = t.gemm_split;
    d["gemm2_pair"] = t.gemm2_pair;
    d["gemm_m64_tails"] = t.gemm_m64_tails;
    d["source"] = t.source;
    return d;
}

/// Device phase-timing buffer of one EP op (allocated on first enable).
/// Rounds reset it with one memset; a snapshot synchronises the stream.
class DebugTiming {
public:
    uint64_t* enable(bool on, torch::Device dev) {
        if (on && !buf_.defined()) {
            buf_ = torch::zeros({ep::kDebugTimeWords}, torch::TensorOptions().dtype(torch::kInt64).device(dev));
        }
        on_ = on;
        if (on) buf_.zero_();
        return ptr();
    }
    bool on() const { return on_; }
    uint64_t* ptr() const { return on_ ? reinterpret_cast<uint64_t*>(buf_.data_ptr<int64_t>()) : nullptr; }
    /// Zeroes every slot on `s` (a memset node when captured in a graph).
    void reset(cudaStream_t s) const {
        if (on_) {
            KIWI_CUDA_CHECK(cudaMemsetAsync(buf_.data_ptr(), 0, ep::kDebugTimeWords * sizeof(uint64_t), s));
        }
    }
    /// {"enabled", "clock", "wall_clock_rate_khz", "time_ticks" (absolute ns, 0 = not recorded),
    ///  "meta", "phase_names", "meta_names"}.
    py::dict snapshot(const std::vector<int32_t>& meta) const {
        cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
        KIWI_CUDA_CHECK(cudaStreamIsCapturing(cur_stream(), &st));
        TORCH_CHECK(st == cudaStreamCaptureStatusNone, "get_debug_timing_snapshot: not allowed during graph capture");
        std::vector<uint64_t> raw(ep::kDebugTimeWords, 0), ticks(ep::kDebugTimeWords, 0);
        if (buf_.defined()) {
            auto h = buf_.cpu();  // ordered after the round's kernels on the current stream
            std::memcpy(raw.data(), h.data_ptr<int64_t>(), raw.size() * sizeof(uint64_t));
            ep::decode_debug_words(raw.data(), ticks.data(), ep::kDebugTimeWords);
        }
        std::vector<int32_t> m(ep::kDebugMetaWords, 0);
        for (size_t i = 0; i < meta.size() && i < m.size(); ++i) m[i] = meta[i];
        py::dict d;
        d["enabled"] = on_;
        d["clock"] = "globaltimer_ns";
        d["wall_clock_rate_khz"] = 1000000;
        d["time_ticks"] = py::cast(ticks);
        d["meta"] = py::cast(m);
        py::list pn, mn;
        for (int i = 0; i < ep::kNumDebugPhases; ++i) pn.append(ep::debug_phase_name(i));
        for (int i = 0; i < ep::kNumDebugMeta; ++i) mn.append(ep::debug_meta_name(i));
        d["phase_names"] = pn;
        d["meta_names"] = mn;
        return d;
    }

private:
    torch::Tensor buf_;
    bool on_ = false;
};

/// Per-source token counts of the last round (ws.slot_tokens) as {received, remote, self}.
std::array<int32_t, 3> recv_token_meta(const torch::Tensor& slot_tokens, const ep::EpConfig& c) {
    auto t = slot_tokens.cpu();
    int32_t all = 0;
    for (int r = 0; r < c.world && r < t.size(0); ++r) all += t[r].item<int32_t>();
    const int32_t self = c.rank < t.size(0) ? t[c.rank].item<int32_t>() : 0;
    return {all, all - self, self};
}

class MoeLayer {
public:
    MoeLayer(p2p::SymmetricHeap& heap, const py::dict& cfg, int64_t ffn, torch::Tensor w13, torch::Tensor w2,
             uint64_t timeout_ns, bool weights_blocked)
        : heap_(heap), cfg_(config_from_dict(cfg)), ffn_(ffn), w13_(w13), w2_(w2), timeout_ns_(timeout_ns),
          blocked_(weights_blocked) {
        TORCH_CHECK(heap.size() >= cfg_.heap_bytes, "symmetric heap too small: need ", cfg_.heap_bytes, " bytes");
        TORCH_CHECK(heap.rank() == cfg_.rank && heap.world() == cfg_.world, "heap rank/world differ from config");
        const int64_t el = cfg_.experts_per_rank;
        // Row-major [E * N, K] or blocked [E * N * K / 64, 64] (kiwi_b200.ops.block_weights).
        const int64_t w13_rows = blocked_ ? el * 2 * ffn * cfg_.hidden / 64 : el * 2 * ffn;
        const int64_t w13_cols = blocked_ ? 64 : cfg_.hidden;
        const int64_t w2_rows = blocked_ ? el * cfg_.hidden * ffn / 64 : el * cfg_.hidden;
        const int64_t w2_cols = blocked_ ? 64 : ffn;
        TORCH_CHECK(w13.is_cuda() && w13.scalar_type() == torch::kBFloat16 && w13.is_contiguous() &&
                        w13.dim() == 2 && w13.size(0) == w13_rows && w13.size(1) == w13_cols,
                    "w13 must be contiguous bf16 [experts_per_rank * 2 * ffn, hidden] (gate/up interleaved by 128), "
                    "or that matrix in the blocked layout with weights_blocked");
        TORCH_CHECK(w2.is_cuda() && w2.scalar_type() == torch::kBFloat16 && w2.is_contiguous() && w2.dim() == 2 &&
                        w2.size(0) == w2_rows && w2.size(1) == w2_cols,
                    "w2 must be contiguous bf16 [experts_per_rank * hidden, ffn], or that matrix in the blocked "
                    "layout with weights_blocked");
        TORCH_CHECK((2 * ffn) % 256 == 0 && cfg_.hidden % 256 == 0 && ffn % 64 == 0 && cfg_.hidden % 64 == 0,
                    "GEMM tiling needs 2*ffn and hidden multiples of 256, ffn of 64");
        auto dev = w13.device();
        auto i32 = torch::TensorOptions().dtype(torch::kInt32).device(dev);
        auto f32 = torch::TensorOptions().dtype(torch::kFloat32).device(dev);
        auto bf = torch::TensorOptions().dtype(torch::kBFloat16).device(dev);
        const int64_t pairs = cfg_.max_pairs();
        epoch_ = torch::zeros({4}, i32);
        done_ = torch::zeros({4}, i32);
        counts_ = torch::zeros({el}, i32);
        cursor_ = torch::zeros({el}, i32);
        offsets_ = torch::zeros({el + 1}, i32);
        tiles1_ = torch::zeros({el + 1}, i32);
        tiles2_ = torch::zeros({el + 1}, i32);
        pair_end_ = torch::zeros({el}, i32);
        split_tiles_ = torch::zeros({4 * (el + 1)}, i32);
        slot_tokens_ = torch::zeros({ep::kMaxTopk}, i32);
        pair_slot_ = torch::zeros({pairs}, i32);
        pair_dst_ = torch::full({pairs}, -1, torch::TensorOptions().dtype(torch::kInt64).device(dev));
        pair_w_ = torch::zeros({pairs}, f32);
        slot_pos_ = torch::full({static_cast<int64_t>(cfg_.slots()) * cfg_.local_per_token()}, -1, i32);
        a_ = torch::zeros({pairs, cfg_.hidden}, bf);
        h_ = torch::zeros({pairs, ffn}, bf);
        y_ = torch::zeros({pairs, cfg_.hidden}, bf);
        error_ = torch::zeros({4}, i32);
        gemm_error_ = torch::zeros({1}, i32);

        ws_.epoch = reinterpret_cast<uint32_t*>(epoch_.data_ptr<int32_t>());
        ws_.done_ctas = reinterpret_cast<uint32_t*>(done_.data_ptr<int32_t>());
        ws_.expert_count = counts_.data_ptr<int32_t>();
        ws_.cursor = cursor_.data_ptr<int32_t>();
        ws_.offsets = offsets_.data_ptr<int32_t>();
        ws_.tiles1 = tiles1_.data_ptr<int32_t>();
        ws_.tiles2 = tiles2_.data_ptr<int32_t>();
        ws_.slot_tokens = slot_tokens_.data_ptr<int32_t>();
        ws_.pair_slot = pair_slot_.data_ptr<int32_t>();
        ws_.pair_dst = pair_dst_.data_ptr<int64_t>();
        ws_.pair_w = pair_w_.data_ptr<float>();
        ws_.slot_pos = slot_pos_.data_ptr<int32_t>();
        ws_.a = reinterpret_cast<__nv_bfloat16*>(a_.data_ptr());
        ws_.error = reinterpret_cast<uint32_t*>(error_.data_ptr<int32_t>());

        tmap_a1_ = gemm::make_tmap_bf16_2d(a_.data_ptr(), pairs, cfg_.hidden, 128);
        tmap_b1_ = gemm::make_tmap_bf16_2d(w13.data_ptr(), w13.size(0), w13.size(1), 256);
        tmap_b1h_ = gemm::make_tmap_bf16_2d(w13.data_ptr(), w13.size(0), w13.size(1), 128);
        tmap_a2_ = gemm::make_tmap_bf16_2d(h_.data_ptr(), pairs, ffn, 128);
        tmap_b2_ = gemm::make_tmap_bf16_2d(w2.data_ptr(), w2.size(0), w2.size(1), 256);
        tmap_b2h_ = gemm::make_tmap_bf16_2d(w2.data_ptr(), w2.size(0), w2.size(1), 128);
        tuning_ = ep::tune(cfg_, gemm::num_sms());
        pair_ = tuning_.gemm_pair;
        pair_auto_ = tuning_.gemm_pair_auto;
        split_ = tuning_.gemm_split;
        pair2_ = tuning_.gemm2_pair;
        m64_ = tuning_.gemm_m64_tails;
        fused_ = tuning_.fused_combine;
        gather_ = tuning_.gather_a;
    }

    // ---- stages (all on the current stream) ----
    void route(torch::Tensor logits, torch::Tensor idx, torch::Tensor w) {
        TORCH_CHECK(logits.scalar_type() == torch::kFloat32 && logits.is_contiguous(), "logits must be fp32");
        TORCH_CHECK(logits.size(1) == cfg_.num_experts, "logits must be [T, num_experts]");
        cudaStream_t s = cur_stream();
        debug_.reset(s);
        routed_ = true;
        ep::launch_route(logits.data_ptr<float>(), static_cast<int>(logits.size(0)), cfg_.num_experts, cfg_.topk,
                         idx.data_ptr<int32_t>(), w.data_ptr<float>(), s, ws_.debug_time);
    }

    void dispatch(torch::Tensor x, torch::Tensor idx, torch::Tensor w) {
        check_tokens(x, idx, w);
        cudaStream_t s = cur_stream();
        if (!routed_) debug_.reset(s);  // a round starts at route() when the layer routes
        routed_ = false;
        tokens_ = static_cast<int>(x.size(0));
        // Rows each local expert expects this round, if every rank sends as many tokens.
        const int64_t rows = static_cast<int64_t>(cfg_.world) * tokens_ * cfg_.topk / cfg_.num_experts;
        use_pair_ = pair_ || (!split_ && pair_auto_ && rows >= ep::kPairMinRows);
        use_split_ = !use_pair_ && split_ && !gathers();
        use_pair2_ = use_pair_ || (pair2_ && !use_split_);
        ep::launch_begin(cfg_, ws_, s);
        ep::launch_dispatch(cfg_, heap_.view(), reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
                            idx.data_ptr<int32_t>(), w.data_ptr<float>(), static_cast<int>(x.size(0)), ws_,
                            tuning_.dispatch_blocks, s);
    }

    void receive() {
        cudaStream_t s = cur_stream();
        // The flag wait runs in a 32-thread kernel of its own, so no kernel that
        // fills the GPU spins on other ranks (two layers' rounds may run on two
        // streams at once).
        ep::launch_wait_flags(cfg_, heap_.view(), ws_, 0, timeout_ns_, s);
        ep::launch_recv_count(cfg_, heap_.view(), ws_, timeout_ns_, s, /*waited=*/true);
        if (use_split_) {
            // Both GEMMs as a 2-SM pass over every expert's full 256-row tiles
            // plus a 1-SM pass over its tail (fewer than 256 rows).
            gemm::build_split_schedule(ws_.expert_count, cfg_.experts_per_rank, static_cast<int>(2 * ffn_),
                                       cfg_.hidden, split_schedule(), s);
        } else {
            // Rows per tile of each GEMM's kernel: the 2-SM kernel takes 256-row
            // tiles; the gathering GEMM1 is a 1-SM kernel.
            const int bm1 = use_pair_ && !gathers() ? 256 : 128;
            const int bm2 = use_pair2_ ? 256 : 128;
            gemm::build_schedule(ws_.expert_count, cfg_.experts_per_rank, static_cast<int>(2 * ffn_), 256,
                                 ws_.offsets, ws_.tiles1, s, bm1);
            gemm::build_schedule(ws_.expert_count, cfg_.experts_per_rank, cfg_.hidden, 256, ws_.offsets, ws_.tiles2, s,
                                 bm2);
        }
        ep::launch_recv_assign(cfg_, heap_.view(), ws_, s, tuning_.recv_blocks);
        if (!gathers()) ep::launch_recv_copy(cfg_, heap_.view(), ws_, s, tuning_.recv_blocks);
    }

    /// GEMM1 reads its A rows in place from the receive buffer (FP8 / NVFP4
    /// dispatch), so the expert-major bf16 copy is skipped.
    bool gathers() const { return gather_ && cfg_.quant != static_cast<int>(ep::Quant::kNone); }

    gemm::SplitSchedule split_schedule() {
        gemm::SplitSchedule ss{};
        ss.offsets = ws_.offsets;
        ss.pair_end = pair_end_.data_ptr<int32_t>();
        ss.pair_tiles1 = split_tiles_.data_ptr<int32_t>();
        ss.tail_tiles1 = ss.pair_tiles1 + (cfg_.experts_per_rank + 1);
        ss.pair_tiles2 = ss.tail_tiles1 + (cfg_.experts_per_rank + 1);
        ss.tail_tiles2 = ss.pair_tiles2 + (cfg_.experts_per_rank + 1);
        return ss;
    }

    /// Runs one GEMM of a split round: the 2-SM pass over full 256-row tiles,
    /// then the 1-SM pass over the tails (rows [pair_end[g], offsets[g + 1])).
    /// `pair(args)` / `tail(args)` launch each pass's kernel.
    template <typename Pair, typename Tail>
    void run_split(const gemm::GroupedArgs& base, const int32_t* pair_tiles, const int32_t* tail_tiles, Pair&& pair,
                   Tail&& tail) {
        gemm::GroupedArgs a = base;
        a.tile_prefix = pair_tiles;
        a.group_end = pair_end_.data_ptr<int32_t>();
        pair(a);
        gemm::GroupedArgs b = base;
        b.tile_prefix = tail_tiles;
        b.group_offset = pair_end_.data_ptr<int32_t>();
        b.group_end = ws_.offsets + 1;
        tail(b);
    }

    void experts() {
        experts_gemm(1);
        experts_gemm(2);
    }

    /// One of the two expert GEMMs (1: gate/up + SwiGLU, 2: down projection;
    /// with fused_combine, GEMM2 also performs the combine's NVLink stores).
    void experts_gemm(int which) {
        TORCH_CHECK(which == 1 || which == 2, "experts_gemm: 1 or 2");
        cudaStream_t s = cur_stream();
        gemm::GroupedArgs g1{};
        g1.group_offset = ws_.offsets;
        g1.tile_prefix = ws_.tiles1;
        g1.num_groups = cfg_.experts_per_rank;
        g1.n = static_cast<int32_t>(2 * ffn_);
        g1.k = cfg_.hidden;
        g1.c = reinterpret_cast<__nv_bfloat16*>(h_.data_ptr());
        g1.ldc = ffn_;
        g1.row_scale = nullptr;
        g1.error = reinterpret_cast<uint32_t*>(gemm_error_.data_ptr<int32_t>());
        g1.max_rows = cfg_.max_pairs();
        g1.m64_tails = m64_ ? 1 : 0;  // read by the 1-SM kernels only
        g1.b_blocked = blocked_ ? 1 : 0;
        g1.span = debug_.on() ? ws_.debug_time + ep::kDebugWordsPerPhase * ep::kPhaseGemm1 : nullptr;
        if (which == 1) {
            if (gathers()) {
                gemm::GatherArgs ga{};
                ga.base = static_cast<const uint8_t*>(heap_.local());
                ga.row_slot = ws_.pair_slot;
                ga.off_row = cfg_.off_row;
                ga.off_scale = cfg_.off_scale;
                ga.row_bytes = cfg_.row_bytes;
                ga.scale_bytes = cfg_.scale_bytes;
                ga.quant = cfg_.quant;
                gemm::grouped_gemm_gather(tmap_b1_, g1, ga, 0, s);
            } else if (use_split_) {
                const gemm::SplitSchedule ss = split_schedule();
                run_split(
                    g1, ss.pair_tiles1, ss.tail_tiles1,
                    [&](const gemm::GroupedArgs& a) { gemm::grouped_gemm_pair(tmap_a1_, tmap_b1h_, a, true, 0, s); },
                    [&](const gemm::GroupedArgs& a) { gemm::grouped_gemm(tmap_a1_, tmap_b1_, a, true, 0, s); });
            } else if (use_pair_) {
                gemm::grouped_gemm_pair(tmap_a1_, tmap_b1h_, g1, /*swiglu=*/true, 0, s);
            } else {
                gemm::grouped_gemm(tmap_a1_, tmap_b1_, g1, /*swiglu=*/true, 0, s);
            }
            return;
        }
        gemm::GroupedArgs g2 = g1;
        g2.tile_prefix = ws_.tiles2;
        g2.n = cfg_.hidden;
        g2.k = static_cast<int32_t>(ffn_);
        g2.c = reinterpret_cast<__nv_bfloat16*>(y_.data_ptr());
        g2.ldc = cfg_.hidden;
        g2.row_scale = ws_.pair_w;
        g2.span = debug_.on() ? ws_.debug_time + ep::kDebugWordsPerPhase * ep::kPhaseGemm2 : nullptr;
        if (fused_) {
            // Fused combine: the epilogue stores every weighted row straight into
            // its token owner's combk slot over NVLink and the last CTA signals.
            gemm::ScatterArgs sc{};
            for (int r = 0; r < cfg_.world; ++r) sc.base[r] = heap_.view().base[r];
            sc.row_dst = ws_.pair_dst;
            sc.done_ctas = ws_.done_ctas + 2;
            sc.epoch = ws_.epoch;
            sc.flag_off = cfg_.combine_flag(cfg_.rank);
            sc.world = cfg_.world;
            if (use_split_) {
                // The 2-SM pass publishes nothing; the tail pass, ordered after it on
                // this stream, signals the round once both passes' rows are out.
                const gemm::SplitSchedule ss = split_schedule();
                gemm::ScatterArgs first = sc;
                first.skip_signal = 1;
                run_split(
                    g2, ss.pair_tiles2, ss.tail_tiles2,
                    [&](const gemm::GroupedArgs& a) { gemm::grouped_gemm_pair_scatter(tmap_a2_, tmap_b2h_, a, first, 0, s); },
                    [&](const gemm::GroupedArgs& a) { gemm::grouped_gemm_scatter(tmap_a2_, tmap_b2_, a, sc, 0, s); });
            } else if (use_pair2_) {
                gemm::grouped_gemm_pair_scatter(tmap_a2_, tmap_b2h_, g2, sc, 0, s);
            } else {
                gemm::grouped_gemm_scatter(tmap_a2_, tmap_b2_, g2, sc, 0, s);
            }
        } else if (use_split_) {
            const gemm::SplitSchedule ss = split_schedule();
            run_split(
                g2, ss.pair_tiles2, ss.tail_tiles2,
                [&](const gemm::GroupedArgs& a) { gemm::grouped_gemm_pair(tmap_a2_, tmap_b2h_, a, false, 0, s); },
                [&](const gemm::GroupedArgs& a) { gemm::grouped_gemm(tmap_a2_, tmap_b2_, a, false, 0, s); });
        } else if (use_pair2_) {
            gemm::grouped_gemm_pair(tmap_a2_, tmap_b2h_, g2, /*swiglu=*/false, 0, s);
        } else {
            gemm::grouped_gemm(tmap_a2_, tmap_b2_, g2, /*swiglu=*/false, 0, s);
        }
    }

    void combine(torch::Tensor idx, torch::Tensor out) {
        cudaStream_t s = cur_stream();
        TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.is_contiguous() && out.dim() == 2 &&
                        out.size(1) == cfg_.hidden && out.device() == w13_.device(),
                    "out must be contiguous bf16 [T, hidden] on the layer's GPU");
        TORCH_CHECK(idx.scalar_type() == torch::kInt32 && idx.is_contiguous() && idx.dim() == 2 &&
                        idx.size(1) == cfg_.topk && idx.size(0) == out.size(0) && out.size(0) <= cfg_.max_tokens,
                    "idx must be the round's contiguous int32 [T, topk] with T = out rows <= max_tokens");
        if (fused_) {
            ep::launch_wait_flags(cfg_, heap_.view(), ws_, 1, timeout_ns_, s);
            ep::launch_combine_recv_fused(cfg_, heap_.view(), idx.data_ptr<int32_t>(), static_cast<int>(out.size(0)),
                                          reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), ws_, timeout_ns_, s,
                                          tuning_.combine_blocks, /*waited=*/true);
            return;
        }
        ep::launch_combine_send(cfg_, heap_.view(), reinterpret_cast<const __nv_bfloat16*>(y_.data_ptr()), ws_,
                                tuning_.combine_blocks, s);
        ep::launch_wait_flags(cfg_, heap_.view(), ws_, 1, timeout_ns_, s);
        ep::launch_combine_recv(cfg_, heap_.view(), idx.data_ptr<int32_t>(), static_cast<int>(out.size(0)),
                                reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), ws_, timeout_ns_, s,
                                tuning_.combine_blocks, nullptr, /*waited=*/true);
    }

    /// The whole layer: x [T, hidden] bf16, idx [T, topk] int32, w [T, topk] fp32 -> out [T, hidden] bf16.
    void forward(torch::Tensor x, torch::Tensor idx, torch::Tensor w, torch::Tensor out) {
        dispatch(x, idx, w);
        receive();
        experts();
        combine(idx, out);
    }

    py::tuple error() const {
        auto e = error_.cpu();
        auto g = gemm_error_.cpu();
        return py::make_tuple(e[0].item<int>(), e[1].item<int>(), e[2].item<int>(), e[3].item<int>(), g[0].item<int>());
    }
    void clear_error() {
        error_.zero_();
        gemm_error_.zero_();
    }

    void set_debug_timing_enabled(bool on) { ws_.debug_time = debug_.enable(on, w13_.device()); }
    bool debug_timing_enabled() const { return debug_.on(); }
    py::dict debug_timing_snapshot() const {
        std::vector<int32_t> m(ep::kNumDebugMeta, 0);
        const auto rt = recv_token_meta(slot_tokens_, cfg_);
        m[ep::kMetaRank] = cfg_.rank;
        m[ep::kMetaWorld] = cfg_.world;
        m[ep::kMetaTokens] = tokens_;
        m[ep::kMetaRecvTokens] = rt[0];
        m[ep::kMetaRecvRemote] = rt[1];
        m[ep::kMetaRecvSelf] = rt[2];
        m[ep::kMetaExpertRows] = offsets_[cfg_.experts_per_rank].item<int32_t>();
        m[ep::kMetaDispatchBlocks] = tuning_.dispatch_blocks;
        m[ep::kMetaRecvBlocks] = tuning_.recv_blocks;
        m[ep::kMetaCombineBlocks] = tuning_.combine_blocks;
        m[ep::kMetaHidden] = cfg_.hidden;
        m[ep::kMetaTopk] = cfg_.topk;
        m[ep::kMetaExpertsPerRank] = cfg_.experts_per_rank;
        m[ep::kMetaQuant] = cfg_.quant;
        m[ep::kMetaFusedCombine] = fused_;
        m[ep::kMetaGatherA] = gathers();
        m[ep::kMetaGemmPair] = use_pair_ ? 1 : (use_split_ ? 2 : (use_pair2_ ? 3 : 0));
        return debug_.snapshot(m);
    }

    py::dict config() const { return config_to_dict(cfg_); }
    torch::Tensor expert_counts() const { return counts_; }
    torch::Tensor expert_offsets() const { return offsets_; }
    torch::Tensor pair_slot() const { return pair_slot_; }
    torch::Tensor pair_weight() const { return pair_w_; }
    torch::Tensor expert_input() const { return a_; }
    torch::Tensor expert_hidden() const { return h_; }
    torch::Tensor expert_output() const { return y_; }
    torch::Tensor epoch() const { return epoch_; }

private:
    void check_tokens(const torch::Tensor& x, const torch::Tensor& idx, const torch::Tensor& w) {
        TORCH_CHECK(x.is_cuda() && x.device() == w13_.device() && idx.device() == x.device() && w.device() == x.device(),
                    "x, idx and w must live on the layer's GPU");
        TORCH_CHECK(x.dim() == 2 && idx.dim() == 2 && w.dim() == 2, "x, idx and w must be 2-D");
        TORCH_CHECK(x.scalar_type() == torch::kBFloat16 && x.is_contiguous() && x.size(1) == cfg_.hidden,
                    "x must be contiguous bf16 [T, hidden]");
        TORCH_CHECK(x.size(0) <= cfg_.max_tokens, "more tokens than max_tokens");
        TORCH_CHECK(idx.scalar_type() == torch::kInt32 && idx.is_contiguous() && idx.size(0) == x.size(0) &&
                        idx.size(1) == cfg_.topk,
                    "idx must be contiguous int32 [T, topk]");
        TORCH_CHECK(w.scalar_type() == torch::kFloat32 && w.is_contiguous() && w.size(0) == x.size(0) &&
                        w.size(1) == cfg_.topk,
                    "w must be contiguous fp32 [T, topk]");
    }

    p2p::SymmetricHeap& heap_;
    ep::EpConfig cfg_;
    int64_t ffn_;
    torch::Tensor w13_, w2_;
    uint64_t timeout_ns_;
    torch::Tensor epoch_, done_, counts_, cursor_, offsets_, tiles1_, tiles2_, slot_tokens_, pair_slot_, pair_w_,
        slot_pos_, a_, h_, y_, error_, gemm_error_, pair_dst_;
    ep::EpWorkspace ws_{};
    CUtensorMap tmap_a1_, tmap_b1_, tmap_a2_, tmap_b2_, tmap_b1h_, tmap_b2h_;
    bool pair_ = false;       // 2-SM GEMMs (256-row tiles only) in every round
    bool split_ = false;      // 2-SM pass over full 256-row tiles + 1-SM pass over the tails, every round
    bool pair_auto_ = true;   // 2-SM GEMMs when a round expects kPairMinRows rows per local expert
    bool use_pair_ = false;   // this round's choices (set by dispatch)
    bool use_split_ = false;
    bool pair2_ = false;      // GEMM2 alone on the 2-SM kernel in every round (GEMM1 stays 1-SM)
    bool m64_ = true;         // 1-SM kernels: M = 64 MMAs on tiles with <= 64 rows of their expert left
    bool blocked_ = false;    // w13 / w2 in the blocked layout (one contiguous 256 x 64 box per TMA load)
    bool use_pair2_ = false;  // this round: GEMM2 on the 2-SM kernel (gemm_pair or gemm2_pair)
    torch::Tensor pair_end_, split_tiles_;
    bool fused_ = true;
    bool gather_ = false;
    ep::EpTuning tuning_{};
    DebugTiming debug_;
    bool routed_ = false;
    int tokens_ = 0;

public:
    bool gather() const { return gather_; }
    void set_gather(bool v) { gather_ = v; }
    bool pair() const { return pair_; }
    void set_pair(bool v) { pair_ = v; }
    bool pair_auto() const { return pair_auto_; }
    void set_pair_auto(bool v) { pair_auto_ = v; }
    bool pair_in_use() const { return use_pair_; }
    bool split_in_use() const { return use_split_; }
    bool split() const { return split_; }
    void set_split(bool v) { split_ = v; }
    bool pair2() const { return pair2_; }
    void set_pair2(bool v) { pair2_ = v; }
    bool pair2_in_use() const { return use_pair2_; }
    bool m64() const { return m64_; }
    void set_m64(bool v) { m64_ = v; }
    bool fused() const { return fused_; }
    py::dict tuning() const { return tuning_dict(tuning_); }
    void set_fused(bool v) { fused_ = v; }
};


/// Transport-only EP op with the reference's dispatch/combine contract.
class Transport {
public:
    Transport(p2p::SymmetricHeap& heap, const py::dict& cfg, uint64_t timeout_ns)
        : heap_(heap), cfg_(config_from_dict(cfg)), timeout_ns_(timeout_ns) {
        TORCH_CHECK(heap.size() >= cfg_.heap_bytes, "symmetric heap too small: need ", cfg_.heap_bytes, " bytes");
        auto dev = torch::Device(torch::kCUDA, c10::cuda::current_device());
        auto i32 = torch::TensorOptions().dtype(torch::kInt32).device(dev);
        auto f32 = torch::TensorOptions().dtype(torch::kFloat32).device(dev);
        auto u8 = torch::TensorOptions().dtype(torch::kUInt8).device(dev);
        const int64_t el = cfg_.experts_per_rank;
        const int64_t slots = static_cast<int64_t>(cfg_.slots());
        epoch_ = torch::zeros({4}, i32);
        done_ = torch::zeros({4}, i32);
        counts_ = torch::zeros({el}, i32);
        cursor_ = torch::zeros({el}, i32);
        slot_tokens_ = torch::zeros({ep::kMaxTopk}, i32);
        error_ = torch::zeros({4}, i32);
        slot_compact_ = torch::full({slots}, -1, i32);
        recv_count_ = torch::zeros({1}, i32);
        rows_ = torch::zeros({slots, cfg_.row_bytes}, u8);
        scales_ = torch::zeros({slots, std::max<int64_t>(cfg_.scale_bytes, 16)}, u8);
        idx_ = torch::zeros({slots, cfg_.topk}, i32);
        w_ = torch::zeros({slots, cfg_.topk}, f32);
        src_pos_ = torch::zeros({slots}, i32);
        ws_.epoch = reinterpret_cast<uint32_t*>(epoch_.data_ptr<int32_t>());
        ws_.done_ctas = reinterpret_cast<uint32_t*>(done_.data_ptr<int32_t>());
        ws_.expert_count = counts_.data_ptr<int32_t>();
        ws_.cursor = cursor_.data_ptr<int32_t>();
        ws_.slot_tokens = slot_tokens_.data_ptr<int32_t>();
        ws_.error = reinterpret_cast<uint32_t*>(error_.data_ptr<int32_t>());
    }

    /// x: bf16 [T, hidden] (quantised here on an FP8 / NVFP4 op), or the
    /// caller's wire bytes [T, row_bytes] (any one-byte dtype) on an FP8 /
    /// NVFP4 op.  scales: the caller's per-token scales [T, ...] (any dtype),
    /// carried as bytes; not allowed with bf16 input on an FP8 / NVFP4 op.
    py::tuple dispatch(torch::Tensor x, torch::Tensor idx, torch::Tensor w, py::object scales, int grid) {
        TORCH_CHECK(x.is_cuda() && x.is_contiguous() && x.dim() == 2, "x must be a contiguous 2-D CUDA tensor");
        TORCH_CHECK(x.size(0) <= cfg_.max_tokens, "more tokens than max_tokens");
        TORCH_CHECK(idx.scalar_type() == torch::kInt32 && idx.is_contiguous() && idx.size(1) == cfg_.topk &&
                        idx.size(0) == x.size(0),
                    "idx must be contiguous int32 [T, topk]");
        TORCH_CHECK(w.scalar_type() == torch::kFloat32 && w.is_contiguous() && w.size(1) == cfg_.topk &&
                        w.size(0) == x.size(0),
                    "w must be contiguous fp32 [T, topk]");
        const void* sp = nullptr;
        int sbytes = 0;
        if (!scales.is_none()) {
            torch::Tensor sc = scales.cast<torch::Tensor>();
            TORCH_CHECK(sc.is_cuda() && sc.is_contiguous() && sc.dim() >= 1 && sc.size(0) == x.size(0),
                        "scales must be a contiguous CUDA tensor with one row per token");
            if (sc.size(0) > 0 && sc.numel() > 0) {
                sbytes = static_cast<int>(sc.numel() / sc.size(0) * sc.element_size());
                TORCH_CHECK(sbytes <= cfg_.scale_bytes, "scales: ", sbytes, " bytes per token exceed the op's ",
                            cfg_.scale_bytes, " (set dispatch_scale_dim / dispatch_scale_type_size)");
                sp = sc.data_ptr();
                scales_in_ = sc;
            }
        }
        cudaStream_t s = cur_stream();
        idx_in_ = idx;
        tokens_ = static_cast<int>(x.size(0));
        debug_.reset(s);
        ep::launch_begin(cfg_, ws_, s);
        if (x.scalar_type() != torch::kBFloat16) {
            TORCH_CHECK(cfg_.quant != static_cast<int>(ep::Quant::kNone),
                        "pre-quantised rows need an FP8 or NVFP4 op (dispatch_quant_format)");
            TORCH_CHECK(x.size(1) * x.element_size() == cfg_.row_bytes, "pre-quantised rows must be [T, ",
                        cfg_.row_bytes, " bytes]");
            ep::launch_dispatch_raw(cfg_, heap_.view(), x.data_ptr(), sp, sbytes, idx.data_ptr<int32_t>(),
                                    w.data_ptr<float>(), tokens_, ws_, grid, s);
        } else {
            TORCH_CHECK(x.size(1) == cfg_.hidden, "x must be bf16 [T, hidden]");
            TORCH_CHECK(sp == nullptr || cfg_.quant == static_cast<int>(ep::Quant::kNone),
                        "an FP8 / NVFP4 op quantises bf16 rows itself and makes their scales; pass pre-quantised "
                        "rows to use your own scales");
            ep::launch_dispatch(cfg_, heap_.view(), reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
                                idx.data_ptr<int32_t>(), w.data_ptr<float>(), tokens_, ws_, grid, s, sp, sbytes);
        }
        ep::launch_recv_count(cfg_, heap_.view(), ws_, timeout_ns_, s);
        ep::launch_recv_compact(cfg_, heap_.view(), ws_, slot_compact_.data_ptr<int32_t>(),
                                recv_count_.data_ptr<int32_t>(), s);
        ep::launch_gather_rows(cfg_, heap_.view(), ws_, slot_compact_.data_ptr<int32_t>(), rows_.data_ptr<uint8_t>(),
                               scales_.data_ptr<uint8_t>(), idx_.data_ptr<int32_t>(), w_.data_ptr<float>(),
                               src_pos_.data_ptr<int32_t>(), s);
        return py::make_tuple(rows_, w_, scales_, idx_, recv_count_);
    }

    /// rows: [>= recv_count, comb_row_bytes] in the combine dtype; weights: fp32
    /// [>= recv_count, topk] or None; out: [>= T, comb_row_bytes]; out_w: fp32
    /// [>= T, topk] (required with weights).
    torch::Tensor combine(torch::Tensor rows, torch::Tensor out, py::object weights, py::object out_w) {
        TORCH_CHECK(rows.is_cuda() && rows.is_contiguous() && rows.dim() == 2 &&
                        rows.size(1) * rows.element_size() == cfg_.comb_row_bytes,
                    "rows must be contiguous [>= recv_count, hidden] in the combine dtype");
        TORCH_CHECK(out.is_cuda() && out.is_contiguous() && out.dim() == 2 && out.size(0) >= tokens_ &&
                        out.size(1) * out.element_size() == cfg_.comb_row_bytes,
                    "out must be contiguous [T, hidden] in the combine dtype");
        TORCH_CHECK(idx_in_.defined(), "combine needs a prior dispatch");
        const float* wp = nullptr;
        float* owp = nullptr;
        if (!weights.is_none()) {
            torch::Tensor wt = weights.cast<torch::Tensor>();
            TORCH_CHECK(wt.scalar_type() == torch::kFloat32 && wt.is_contiguous() && wt.dim() == 2 &&
                            wt.size(1) == cfg_.topk && wt.size(0) >= rows.size(0),
                        "weights must be contiguous fp32 [rows, topk]");
            TORCH_CHECK(!out_w.is_none(), "weights need an output weight buffer");
            torch::Tensor ow = out_w.cast<torch::Tensor>();
            TORCH_CHECK(ow.scalar_type() == torch::kFloat32 && ow.is_contiguous() && ow.dim() == 2 &&
                            ow.size(1) == cfg_.topk && ow.size(0) >= tokens_,
                        "out_weights must be contiguous fp32 [T, topk]");
            wp = wt.data_ptr<float>();
            owp = ow.data_ptr<float>();
            weights_in_ = wt;
        }
        cudaStream_t s = cur_stream();
        ep::launch_combine_rows(cfg_, heap_.view(), rows.data_ptr(), wp, src_pos_.data_ptr<int32_t>(),
                                recv_count_.data_ptr<int32_t>(), ws_, s);
        ep::launch_combine_recv(cfg_, heap_.view(), idx_in_.data_ptr<int32_t>(), tokens_, out.data_ptr(), ws_,
                                timeout_ns_, s, 0, owp);
        return out;
    }

    py::tuple error() const {
        auto e = error_.cpu();
        return py::make_tuple(e[0].item<int>(), e[1].item<int>(), e[2].item<int>(), e[3].item<int>());
    }
    torch::Tensor src_token_pos() const { return src_pos_; }
    py::dict config() const { return config_to_dict(cfg_); }

    void set_debug_timing_enabled(bool on) { ws_.debug_time = debug_.enable(on, epoch_.device()); }
    bool debug_timing_enabled() const { return debug_.on(); }
    py::dict debug_timing_snapshot() const {
        std::vector<int32_t> m(ep::kNumDebugMeta, 0);
        const auto rt = recv_token_meta(slot_tokens_, cfg_);
        m[ep::kMetaRank] = cfg_.rank;
        m[ep::kMetaWorld] = cfg_.world;
        m[ep::kMetaTokens] = tokens_;
        m[ep::kMetaRecvTokens] = rt[0];
        m[ep::kMetaRecvRemote] = rt[1];
        m[ep::kMetaRecvSelf] = rt[2];
        m[ep::kMetaExpertRows] = recv_count_.cpu()[0].item<int32_t>();
        m[ep::kMetaHidden] = cfg_.hidden;
        m[ep::kMetaTopk] = cfg_.topk;
        m[ep::kMetaExpertsPerRank] = cfg_.experts_per_rank;
        m[ep::kMetaQuant] = cfg_.quant;
        return debug_.snapshot(m);
    }

private:
    p2p::SymmetricHeap& heap_;
    ep::EpConfig cfg_;
    uint64_t timeout_ns_;
    int tokens_ = 0;
    torch::Tensor epoch_, done_, counts_, cursor_, slot_tokens_, error_, slot_compact_, recv_count_, rows_, scales_,
        idx_, w_, src_pos_, idx_in_, scales_in_, weights_in_;
    ep::EpWorkspace ws_{};
    DebugTiming debug_;
};

}  // namespace

void register_ep(py::module_& m) {
    auto e = m.def_submodule("ep", "kiwi::ep (expert-parallel MoE)");
    e.attr("MAX_TOPK") = ep::kMaxTopk;
    e.attr("DEBUG_TIME_WORDS") = ep::kDebugTimeWords;
    e.attr("DEBUG_WORDS_PER_PHASE") = ep::kDebugWordsPerPhase;
    {
        py::list pn, mn;
        for (int i = 0; i < ep::kNumDebugPhases; ++i) pn.append(ep::debug_phase_name(i));
        for (int i = 0; i < ep::kNumDebugMeta; ++i) mn.append(ep::debug_meta_name(i));
        e.attr("DEBUG_PHASES") = pn;
        e.attr("DEBUG_META") = mn;
    }
    e.def("dispatch_grid", &ep::dispatch_grid, py::arg("tokens"), py::arg("tuned"), py::arg("sms"),
          "Blocks the dispatch kernel launches for `tokens` tokens (tuned > 0: that many).");
    e.def("decode_debug_words",
          [](const std::vector<uint64_t>& raw) {
              std::vector<uint64_t> out(raw.size(), 0);
              ep::decode_debug_words(raw.data(), out.data(), static_cast<int>(raw.size()));
              return out;
          },
          "Raw phase words (start slots hold ~t) -> absolute ns, 0 = not recorded.");
    e.def("finalize_config", [](const py::dict& d) { return config_to_dict(config_from_dict(d)); });
    e.def("tune", [](const py::dict& d, int sms, py::object env) {
              std::string ev;
              if (!env.is_none()) ev = env.cast<std::string>();
              return tuning_dict(ep::tune(config_from_dict(d), sms, env.is_none() ? nullptr : ev.c_str()));
          },
          py::arg("config"), py::arg("sms"), py::arg("env") = py::none(),
          "B200 launch tuning of an EP configuration (env: a KIWI_EP_TUNING override string).");
    e.def("route",
          [](torch::Tensor logits, int topk, torch::Tensor idx, torch::Tensor w) {
              ep::launch_route(logits.data_ptr<float>(), static_cast<int>(logits.size(0)),
                               static_cast<int>(logits.size(1)), topk, idx.data_ptr<int32_t>(), w.data_ptr<float>(),
                               cur_stream());
          },
          "Top-k routing with softmax over the selected logits (fp32 logits [T, E]).");
    py::class_<Transport>(e, "Transport")
        .def(py::init<p2p::SymmetricHeap&, const py::dict&, uint64_t>(), py::arg("heap"), py::arg("config"),
             py::arg("timeout_ns") = 5000000000ull, py::keep_alive<1, 2>())
        .def("dispatch", &Transport::dispatch, py::arg("x"), py::arg("idx"), py::arg("w"),
             py::arg("scales") = py::none(), py::arg("grid") = 0)
        .def("combine", &Transport::combine, py::arg("rows"), py::arg("out"), py::arg("weights") = py::none(),
             py::arg("out_weights") = py::none())
        .def("error", &Transport::error)
        .def("set_debug_timing_enabled", &Transport::set_debug_timing_enabled, py::arg("enabled"))
        .def_property_readonly("debug_timing_enabled", &Transport::debug_timing_enabled)
        .def("get_debug_timing_snapshot", &Transport::debug_timing_snapshot)
        .def_property_readonly("src_token_pos", &Transport::src_token_pos)
        .def_property_readonly("config", &Transport::config);
    py::class_<MoeLayer>(e, "MoeLayer")
        .def(py::init<p2p::SymmetricHeap&, const py::dict&, int64_t, torch::Tensor, torch::Tensor, uint64_t, bool>(),
             py::arg("heap"), py::arg("config"), py::arg("ffn"), py::arg("w13"), py::arg("w2"),
             py::arg("timeout_ns") = 5000000000ull, py::arg("weights_blocked") = false, py::keep_alive<1, 2>())
        .def("route", &MoeLayer::route)
        .def("dispatch", &MoeLayer::dispatch)
        .def("receive", &MoeLayer::receive)
        .def("experts", &MoeLayer::experts)
        .def("experts_gemm", &MoeLayer::experts_gemm, py::arg("which"))
        .def("combine", &MoeLayer::combine)
        .def("forward", &MoeLayer::forward)
        .def("error", &MoeLayer::error)
        .def("clear_error", &MoeLayer::clear_error)
        .def("set_debug_timing_enabled", &MoeLayer::set_debug_timing_enabled, py::arg("enabled"),
             "Per-kernel %globaltimer spans of every round (first block start, last warp end, flag waits).")
        .def_property_readonly("debug_timing_enabled", &MoeLayer::debug_timing_enabled)
        .def("get_debug_timing_snapshot", &MoeLayer::debug_timing_snapshot,
             "Synchronises the current stream and returns the last round's phase stamps.")
        .def_property_readonly("config", &MoeLayer::config)
        .def_property_readonly("expert_counts", &MoeLayer::expert_counts)
        .def_property_readonly("expert_offsets", &MoeLayer::expert_offsets)
        .def_property_readonly("pair_slot", &MoeLayer::pair_slot)
        .def_property_readonly("pair_weight", &MoeLayer::pair_weight)
        .def_property_readonly("expert_input", &MoeLayer::expert_input)
        .def_property_readonly("expert_hidden", &MoeLayer::expert_hidden)
        .def_property_readonly("expert_output", &MoeLayer::expert_output)
        .def_property_readonly("epoch", &MoeLayer::epoch)
        .def_property("gemm_pair_auto", &MoeLayer::pair_auto, &MoeLayer::set_pair_auto,
                      "Run the 2-SM GEMMs in rounds whose expected rows per local expert reach 4096 (default on).")
        .def_property("gemm_split", &MoeLayer::split, &MoeLayer::set_split,
                      "Split both GEMMs into a 2-SM pass over every expert's full 256-row tiles and a 1-SM pass "
                      "over its tail (opt-in: measured slower under the power cap).")
        .def_property_readonly("gemm_pair_in_use", &MoeLayer::pair_in_use,
                               "Whether the last dispatched round runs the 2-SM GEMMs alone (gemm_pair).")
        .def_property_readonly("gemm_split_in_use", &MoeLayer::split_in_use,
                               "Whether the last dispatched round runs the split (2-SM + 1-SM tail) GEMMs.")
        .def_property("gemm2_pair", &MoeLayer::pair2, &MoeLayer::set_pair2,
                      "Run the down projection (GEMM2, with its combine epilogue) on the 2-SM kernel and the "
                      "gate/up GEMM on the 1-SM kernel in every round (opt-in).")
        .def_property("gemm_m64_tails", &MoeLayer::m64, &MoeLayer::set_m64,
                      "1-SM GEMM tiles with at most 64 rows of their expert left run M = 64 MMAs (default on; the "
                      "result is bit-identical).")
        .def_property_readonly("gemm2_pair_in_use", &MoeLayer::pair2_in_use,
                               "Whether the last dispatched round runs GEMM2 on the 2-SM kernel.")
        .def_property("gemm_pair", &MoeLayer::pair, &MoeLayer::set_pair,
                      "Use the 2-SM (256-row tile) grouped GEMMs in every round (off by default; gemm_pair_auto "
                      "picks them per round).")
        .def_property_readonly("tuning", &MoeLayer::tuning, "Launch tuning in effect (B200 table + KIWI_EP_TUNING).")
        .def_property("gather_a", &MoeLayer::gather, &MoeLayer::set_gather,
                      "GEMM1 gathers and dequantises its A rows from the receive buffer (FP8 / NVFP4 dispatch; "
                      "opt-in: measured slower than the default, where a receive kernel first writes "
                      "expert-major bf16 rows that TMA loads).")
        .def_property("fused_combine", &MoeLayer::fused, &MoeLayer::set_fused,
                      "GEMM2 epilogue stores rows over NVLink into the token owners' top-k slots (default); "
                      "False: GEMM2 to local memory, then combine send + receive kernels.");
}
