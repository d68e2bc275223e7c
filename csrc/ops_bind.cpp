// Python bindings of the sm_100a compute ops (kiwi_b200._C.ops).
#include <ATen/cuda/CUDAContext.h>
#include <algorithm>
#include <c10/cuda/CUDAGuard.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <torch/extension.h>

#include "kiwi/ep/kernels.hpp"
#include "kiwi/gemm/grouped_gemm.hpp"
#include "kiwi/ops/quant.hpp"
#include "kiwi/ops/rows.hpp"

namespace py = pybind11;
using namespace kiwi;

namespace {

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

/// A grouped GEMM bound to fixed A and B buffers (their tensor maps are built once).
class GroupedGemm {
public:
    GroupedGemm(torch::Tensor a, torch::Tensor b, int64_t num_groups, bool b_blocked)
        : a_(a), b_(b), num_groups_(static_cast<int>(num_groups)), b_blocked_(b_blocked) {
        TORCH_CHECK(a.is_cuda() && b.is_cuda(), "A and B must be CUDA tensors");
        TORCH_CHECK(a.scalar_type() == torch::kBFloat16 && b.scalar_type() == torch::kBFloat16, "bf16 only");
        TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.is_contiguous() && b.is_contiguous(), "2-D contiguous");
        k_ = static_cast<int>(a.size(1));
        if (b_blocked) {
            // [G * N * K / 64, 64]: one contiguous 256 x 64 box per (group, n-tile, k-block).
            TORCH_CHECK(b.size(1) == 64 && k_ % 64 == 0 && (b.size(0) * 64) % (num_groups * k_) == 0,
                        "blocked B must be [num_groups * N * K / 64, 64]");
            n_ = static_cast<int>(b.size(0) * 64 / (num_groups * k_));
        } else {
            TORCH_CHECK(a.size(1) == b.size(1), "A and B must share K");
            TORCH_CHECK(b.size(0) % num_groups == 0, "B rows must be num_groups * N");
            n_ = static_cast<int>(b.size(0) / num_groups);
        }
        TORCH_CHECK(k_ % 64 == 0 && n_ % 256 == 0, "K % 64 == 0 and N % 256 == 0 required");
        const int64_t b_cols = b_blocked ? 64 : k_;
        tmap_a_ = gemm::make_tmap_bf16_2d(a.data_ptr(), a.size(0), k_, 128);
        tmap_b_ = gemm::make_tmap_bf16_2d(b.data_ptr(), b.size(0), b_cols, 256);
        tmap_b_half_ = gemm::make_tmap_bf16_2d(b.data_ptr(), b.size(0), b_cols, 128);
        if (k_ % 32 == 0 && !b_blocked) {
            tmap_a32_ = gemm::make_tmap_bf16_2d(a.data_ptr(), a.size(0), k_, 128, 32);
            tmap_b32_ = gemm::make_tmap_bf16_2d(b.data_ptr(), b.size(0), k_, 256, 32);
        }
        auto iopts = torch::TensorOptions().dtype(torch::kInt32).device(a.device());
        offsets_ = torch::zeros({num_groups_ + 1}, iopts);
        tile_prefix_ = torch::zeros({num_groups_ + 1}, iopts);
        error_ = torch::zeros({1}, iopts);
    }

    /// counts: int32[G] rows per group (device); out: bf16 [rows, N] or [rows, N/2] with swiglu.
    void run(torch::Tensor counts, torch::Tensor out, bool swiglu, py::object row_scale, int grid, bool pair,
             py::object trace, int bk, bool m64) {
        TORCH_CHECK(bk == 64 || bk == 32 || bk == 128, "bk must be 64, 32 or 128");
        TORCH_CHECK(bk == 64 || !pair, "bk = 32 and 128 are 1-SM variants");
        TORCH_CHECK(bk == 64 || !b_blocked_, "the blocked B layout runs with bk = 64 only");
        TORCH_CHECK(bk != 128 || k_ % 128 == 0, "bk = 128 needs K a multiple of 128");
        TORCH_CHECK(counts.is_cuda() && counts.scalar_type() == torch::kInt32 && counts.numel() == num_groups_,
                    "counts must be int32[num_groups] on the device");
        TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.is_contiguous(), "out must be contiguous bf16");
        TORCH_CHECK(out.size(1) == (swiglu ? n_ / 2 : n_), "out has the wrong number of columns");
        TORCH_CHECK(out.size(0) >= a_.size(0), "out needs at least as many rows as A");
        const float* rs = nullptr;
        if (!row_scale.is_none()) {
            torch::Tensor t = row_scale.cast<torch::Tensor>();
            TORCH_CHECK(t.scalar_type() == torch::kFloat32 && t.is_cuda(), "row_scale must be fp32 CUDA");
            rs = t.data_ptr<float>();
            row_scale_ref_ = t;
        }
        cudaStream_t s = cur_stream();
        gemm::build_schedule(counts.data_ptr<int32_t>(), num_groups_, n_, 256, offsets_.data_ptr<int32_t>(),
                             tile_prefix_.data_ptr<int32_t>(), s, pair ? 256 : 128);
        gemm::GroupedArgs args{};
        args.group_offset = offsets_.data_ptr<int32_t>();
        args.tile_prefix = tile_prefix_.data_ptr<int32_t>();
        args.num_groups = num_groups_;
        args.n = n_;
        args.k = k_;
        args.c = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
        args.ldc = out.size(1);
        args.row_scale = rs;
        args.error = reinterpret_cast<uint32_t*>(error_.data_ptr<int32_t>());
        args.max_rows = out.size(0);
        args.m64_tails = !pair && m64;
        args.b_blocked = b_blocked_ ? 1 : 0;
        if (!trace.is_none()) {
            torch::Tensor t = trace.cast<torch::Tensor>();
            TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kInt64 && t.is_contiguous() && !pair,
                        "trace must be a contiguous int64 CUDA tensor (1-SM kernel only)");
            args.trace = reinterpret_cast<uint64_t*>(t.data_ptr<int64_t>());
            args.trace_capacity = t.numel() / gemm::kTraceSlots;
            trace_ref_ = t;
        }
        if (bk == 32) {
            gemm::grouped_gemm_bk32(tmap_a32_, tmap_b32_, args, swiglu, grid, s);
        } else if (bk == 128) {
            gemm::grouped_gemm_bk128(tmap_a_, tmap_b_, args, swiglu, grid, s);
        } else if (pair) {
            gemm::grouped_gemm_pair(tmap_a_, tmap_b_half_, args, swiglu, grid, s);
        } else {
            gemm::grouped_gemm(tmap_a_, tmap_b_, args, swiglu, grid, s);
        }
    }

    torch::Tensor offsets() const { return offsets_; }
    torch::Tensor tile_prefix() const { return tile_prefix_; }
    torch::Tensor error() const { return error_; }

private:
    torch::Tensor a_, b_, offsets_, tile_prefix_, error_, row_scale_ref_, trace_ref_;
    int num_groups_, n_, k_;
    bool b_blocked_ = false;
    CUtensorMap tmap_a_, tmap_b_, tmap_b_half_, tmap_a32_, tmap_b32_;
};

void check_rows_tensor(const torch::Tensor& t, const char* what) {
    TORCH_CHECK(t.is_cuda() && t.dim() == 2 && t.is_contiguous(), what, " must be a contiguous 2-D CUDA tensor");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, what, " must start on a 16-byte boundary");
}

const int32_t* index_ptr(const py::object& idx, int64_t rows, const torch::Device& dev, const char* what) {
    if (idx.is_none()) return nullptr;
    torch::Tensor t = idx.cast<torch::Tensor>();
    TORCH_CHECK(t.device() == dev && t.scalar_type() == torch::kInt32 && t.is_contiguous() && t.numel() >= rows,
                what, " must be a contiguous int32 tensor on the rows' device with at least `rows` entries");
    return t.data_ptr<int32_t>();
}

void check_error_word(const torch::Tensor& e, const torch::Device& dev) {
    TORCH_CHECK(e.device() == dev && e.scalar_type() == torch::kInt32 && e.numel() >= 1,
                "error must be an int32 tensor on the rows' device");
}

void rows_copy_py(torch::Tensor src, torch::Tensor dst, py::object src_idx, py::object dst_idx, int64_t rows,
                  torch::Tensor error, int grid) {
    check_rows_tensor(src, "src");
    check_rows_tensor(dst, "dst");
    TORCH_CHECK(src.device() == dst.device(), "src and dst must be on one device");
    const int64_t row_bytes = src.size(1) * src.element_size();
    TORCH_CHECK(row_bytes == dst.size(1) * dst.element_size() && row_bytes % 16 == 0,
                "src and dst rows must have the same size, a multiple of 16 bytes");
    if (rows < 0) {
        if (!src_idx.is_none()) rows = src_idx.cast<torch::Tensor>().numel();
        else if (!dst_idx.is_none()) rows = dst_idx.cast<torch::Tensor>().numel();
        else rows = std::min(src.size(0), dst.size(0));
    }
    TORCH_CHECK(!src_idx.is_none() || rows <= src.size(0), "rows exceeds src without a source index");
    TORCH_CHECK(!dst_idx.is_none() || rows <= dst.size(0), "rows exceeds dst without a destination index");
    const c10::cuda::CUDAGuard guard(src.device());
    check_error_word(error, src.device());
    ops::rows_copy(src.data_ptr(), dst.data_ptr(), index_ptr(src_idx, rows, src.device(), "src_idx"),
                   index_ptr(dst_idx, rows, src.device(), "dst_idx"), rows, row_bytes, src.size(0), dst.size(0),
                   reinterpret_cast<uint32_t*>(error.data_ptr<int32_t>()), grid, cur_stream());
}

void rows_accumulate_py(torch::Tensor src, torch::Tensor out, torch::Tensor map, torch::Tensor error, int grid) {
    check_rows_tensor(src, "src");
    check_rows_tensor(out, "out");
    TORCH_CHECK(src.scalar_type() == torch::kBFloat16 && out.scalar_type() == torch::kBFloat16, "bf16 rows only");
    TORCH_CHECK(src.size(1) == out.size(1) && src.size(1) % 8 == 0, "src and out share hidden, a multiple of 8");
    TORCH_CHECK(map.device() == src.device() && out.device() == src.device() && map.scalar_type() == torch::kInt32 &&
                    map.dim() == 2 && map.is_contiguous() && map.size(0) <= out.size(0),
                "map must be a contiguous int32 [tokens, k] tensor on src's device, tokens <= out rows");
    TORCH_CHECK(map.size(1) >= 1 && map.size(1) <= ops::kRowsMaxK, "k must be in [1, ", ops::kRowsMaxK, "]");
    const c10::cuda::CUDAGuard guard(src.device());
    check_error_word(error, src.device());
    ops::rows_accumulate_bf16(src.data_ptr(), out.data_ptr(), map.data_ptr<int32_t>(), map.size(0),
                              static_cast<int>(map.size(1)), src.size(1), src.size(0),
                              reinterpret_cast<uint32_t*>(error.data_ptr<int32_t>()), grid, cur_stream());
}

}  // namespace

void register_ops(py::module_& m) {
    auto o = m.def_submodule("ops", "sm_100a compute kernels");
    py::class_<GroupedGemm>(o, "GroupedGemm")
        .def(py::init<torch::Tensor, torch::Tensor, int64_t, bool>(), py::arg("a"), py::arg("b"),
             py::arg("num_groups"), py::arg("b_blocked") = false,
             "b: [num_groups * N, K] row-major, or with b_blocked the layout of kiwi_b200.ops.block_weights "
             "([num_groups * N * K / 64, 64], one contiguous 256 x 64 box per group, n-tile and k-block).")
        .def("run", &GroupedGemm::run, py::arg("counts"), py::arg("out"), py::arg("swiglu") = false,
             py::arg("row_scale") = py::none(), py::arg("grid") = 0, py::arg("pair") = false,
             py::arg("trace") = py::none(), py::arg("bk") = 64, py::arg("m64") = true,
             "Grouped GEMM on the current stream.  bk: K columns per pipeline stage of the 1-SM kernel (64: "
             "4 x 48 KB stages, the default; 32: 64-byte swizzle, 9 stages; 128: two 64-column boxes per operand, "
             "2 x 96 KB stages).  All three issue the same K = 16 MMAs in the same order.  m64 (1-SM kernels, on by "
             "default): tiles with at most 64 rows of their group left run M = 64 MMAs; the result is "
             "bit-identical.")
        .def_property_readonly("offsets", &GroupedGemm::offsets)
        .def_property_readonly("tile_prefix", &GroupedGemm::tile_prefix)
        .def_property_readonly("error", &GroupedGemm::error);
    o.def("gemm_kernel_info", [](bool swiglu) {
        const auto i = gemm::gemm_kernel_info(swiglu);
        return py::make_tuple(i.local_bytes, i.registers, i.smem_bytes);
    });
    o.def("gemm_pair_kernel_info", [](bool swiglu) {
        const auto i = gemm::gemm_pair_kernel_info(swiglu);
        return py::make_tuple(i.local_bytes, i.registers, i.smem_bytes);
    });
    o.def("gemm_scatter_kernel_info", [](bool pair) {
        const auto i = pair ? gemm::gemm_pair_scatter_kernel_info() : gemm::gemm_scatter_kernel_info();
        return py::make_tuple(i.local_bytes, i.registers, i.smem_bytes);
    }, py::arg("pair") = false, "(local bytes, registers, shared bytes) of the NVLink scatter GEMM (1-SM or 2-SM).");
    o.def("num_sms", &gemm::num_sms);
    o.def(
        "quant_fp8",
        [](torch::Tensor x) {
            TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.dim() == 2 && x.is_contiguous(),
                        "x must be a contiguous bf16 [rows, hidden] CUDA tensor");
            TORCH_CHECK(x.size(1) % 128 == 0, "hidden must be a multiple of 128");
            TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0, "x must start on a 16-byte boundary");
            const c10::cuda::CUDAGuard guard(x.device());
            auto opts = torch::TensorOptions().device(x.device());
            torch::Tensor codes = torch::empty({x.size(0), x.size(1)}, opts.dtype(torch::kFloat8_e4m3fn));
            torch::Tensor scales = torch::empty({x.size(0), x.size(1) / 128}, opts.dtype(torch::kFloat32));
            ops::quant_fp8_rows(x.data_ptr(), codes.data_ptr(), scales.data_ptr<float>(), x.size(0),
                                static_cast<int>(x.size(1)), cur_stream());
            return py::make_tuple(codes, scales);
        },
        py::arg("x"),
        "1x128 FP8 e4m3 quantisation of bf16 rows with the dispatch kernel's arithmetic: (codes, fp32 scales).");
    o.def(
        "quant_nvfp4",
        [](torch::Tensor x) {
            TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.dim() == 2 && x.is_contiguous(),
                        "x must be a contiguous bf16 [rows, hidden] CUDA tensor");
            TORCH_CHECK(x.size(1) % 16 == 0, "hidden must be a multiple of 16");
            TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0, "x must start on a 16-byte boundary");
            const c10::cuda::CUDAGuard guard(x.device());
            const int hidden = static_cast<int>(x.size(1));
            auto opts = torch::TensorOptions().device(x.device()).dtype(torch::kUInt8);
            torch::Tensor codes = torch::empty({x.size(0), hidden / 2}, opts);
            torch::Tensor scales = torch::empty({x.size(0), ops::nvfp4_scale_bytes(hidden)}, opts);
            ops::quant_nvfp4_rows(x.data_ptr(), codes.data_ptr(), scales.data_ptr(), x.size(0), hidden,
                                  cur_stream());
            return py::make_tuple(codes, scales);
        },
        py::arg("x"),
        "NVFP4 quantisation of bf16 rows into the NVLink dispatch's wire bytes: (packed e2m1 codes uint8 "
        "[rows, hidden / 2], scale bytes uint8 [rows, S]: fp32 row scale then e4m3 block scales).");
    o.def(
        "route_topk",
        [](torch::Tensor logits, int64_t topk) {
            TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == torch::kFloat32 && logits.dim() == 2 &&
                            logits.is_contiguous(),
                        "logits must be a contiguous fp32 [tokens, experts] CUDA tensor");
            TORCH_CHECK(topk >= 1 && topk <= logits.size(1), "topk must be in [1, experts]");
            const c10::cuda::CUDAGuard guard(logits.device());
            auto opts = torch::TensorOptions().device(logits.device());
            torch::Tensor idx = torch::empty({logits.size(0), topk}, opts.dtype(torch::kInt32));
            torch::Tensor w = torch::empty({logits.size(0), topk}, opts.dtype(torch::kFloat32));
            ep::launch_route(logits.data_ptr<float>(), static_cast<int>(logits.size(0)),
                             static_cast<int>(logits.size(1)), static_cast<int>(topk), idx.data_ptr<int32_t>(),
                             w.data_ptr<float>(), cur_stream());
            return py::make_tuple(idx, w);
        },
        py::arg("logits"), py::arg("topk"),
        "Top-k experts per token and the softmax over their logits (the EP layer's routing kernel): "
        "(idx int32 [T, k], weights fp32 [T, k]) on the current stream.");
    o.def("rows_copy", &rows_copy_py, py::arg("src"), py::arg("dst"), py::arg("src_idx") = py::none(),
          py::arg("dst_idx") = py::none(), py::arg("rows") = -1, py::arg("error"), py::arg("grid") = 0,
          "dst[dst_idx[i]] = src[src_idx[i]] (identity where an index is None), i < rows; negative indices skip "
          "the row, out-of-range ones set bits of `error` (int32[1]) and skip it.  Current stream.");
    o.def("rows_accumulate", &rows_accumulate_py, py::arg("src"), py::arg("out"), py::arg("map"), py::arg("error"),
          py::arg("grid") = 0,
          "out[t] = sum_j src[map[t, j]] (bf16 rows, fp32 sums); negative entries are skipped.  Current stream.");
}
