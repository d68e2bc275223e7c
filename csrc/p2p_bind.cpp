// Python bindings of kiwi::p2p: symmetric heap, FD exchange, P2P kernels.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAStream.h>
#include <pybind11/functional.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <torch/extension.h>
#include <unistd.h>

#include "kiwi/p2p/collectives.cuh"
#include "kiwi/p2p/context.hpp"
#include "kiwi/p2p/heap.hpp"
#include "kiwi/p2p/p2p_ops.hpp"

namespace py = pybind11;
using namespace kiwi;
using namespace kiwi::p2p;

namespace {
cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

torch::Tensor view_tensor(void* base, uint64_t heap_size, int device, uint64_t offset, std::vector<int64_t> shape,
                          torch::Dtype dtype) {
    int64_t numel = 1;
    for (auto d : shape) numel *= d;
    const uint64_t bytes = static_cast<uint64_t>(numel) * c10::elementSize(dtype);
    if (offset + bytes > heap_size) throw kiwi::error("kiwi::p2p: tensor view exceeds the heap");
    auto opts = torch::TensorOptions().dtype(dtype).device(torch::kCUDA, device);
    return torch::from_blob(static_cast<uint8_t*>(base) + offset, shape, opts);
}

uint64_t* u64_ptr(const torch::Tensor& t) {
    TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kInt64, "expected a CUDA int64 tensor");
    return reinterpret_cast<uint64_t*>(t.data_ptr<int64_t>());
}
uint32_t* u32_ptr(const torch::Tensor& t) {
    TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kInt32, "expected a CUDA int32 tensor");
    return reinterpret_cast<uint32_t*>(t.data_ptr<int32_t>());
}
}  // namespace

void register_p2p(py::module_& m) {
    auto p = m.def_submodule("p2p", "kiwi::p2p (NVLink peer memory)");
    p.attr("MAX_RANKS") = kMaxRanks;
    p.def("exchange_fds", &exchange_fds, py::arg("job"), py::arg("rank"), py::arg("world"), py::arg("fd"),
          py::arg("timeout_s") = 60.0, py::call_guard<py::gil_scoped_release>());
    p.def("broadcast_fd", &broadcast_fd, py::arg("job"), py::arg("rank"), py::arg("world"), py::arg("root"),
          py::arg("fd"), py::arg("timeout_s") = 60.0, py::call_guard<py::gil_scoped_release>());
    p.def("multicast_supported", &SymmetricHeap::multicast_supported);
    p.def("coll_ingress_bytes", [](int world) { return coll_ingress_bytes(world); });
    p.def("heap_range_ok", &heap_range_ok, py::arg("world"), py::arg("limit"), py::arg("rank"), py::arg("off"),
          py::arg("bytes"), "The checked mode's range rule: rank in [0, world), [off, off + bytes) in [0, limit).");
    py::enum_<CheckSite>(p, "CheckSite")
        .value("PUT", kCheckPut)
        .value("GET", kCheckGet)
        .value("SIGNAL", kCheckSignal)
        .value("LL8", kCheckLl8)
        .value("MULTICAST", kCheckMulticast);
    p.def("grid_barrier_test",
          [](uint32_t blocks, uint32_t rounds, uint64_t timeout_ns) {
              auto opts = torch::TensorOptions().device(torch::kCUDA, c10::cuda::current_device());
              auto word = torch::zeros({1}, opts.dtype(torch::kInt64));
              auto data = torch::zeros({static_cast<int64_t>(blocks)}, opts.dtype(torch::kInt32));
              auto status = torch::zeros({2}, opts.dtype(torch::kInt32));
              auto el = torch::zeros({1}, opts.dtype(torch::kInt64));
              launch_grid_barrier_test(reinterpret_cast<unsigned long long*>(word.data_ptr<int64_t>()),
                                       u32_ptr(data), blocks, rounds, u32_ptr(status), timeout_ns, u64_ptr(el),
                                       cur_stream());
              KIWI_CUDA_CHECK(cudaStreamSynchronize(cur_stream()));
              py::dict d;
              d["status"] = status[0].item<int32_t>();
              d["info"] = status[1].item<int32_t>();
              d["elapsed_ns"] = el[0].item<int64_t>();
              d["word"] = word[0].item<int64_t>();
              return d;
          },
          py::arg("blocks"), py::arg("rounds"), py::arg("timeout_ns") = 2000000000ull);

    py::class_<CompletionCounter>(p, "CompletionCounter",
                                  "64-bit counter in mapped pinned memory: host signal(), kernel poll.")
        .def(py::init([](bool host_only) {
                 return std::make_unique<CompletionCounter>(host_only ? queue::MemKind::kHost
                                                                      : queue::MemKind::kMappedPinned);
             }),
             py::arg("host_only") = false)
        .def("signal", &CompletionCounter::signal, py::arg("n") = 1)
        .def("get", &CompletionCounter::get)
        .def("set", &CompletionCounter::set)
        .def("wait_kernel",
             [](CompletionCounter& c, uint32_t steps, torch::Tensor seen, torch::Tensor status, uint64_t timeout_ns) {
                 if (seen.numel() < steps) throw kiwi::error("wait_kernel: seen needs steps entries");
                 launch_counter_wait(c.device_view(), steps, u64_ptr(seen), u32_ptr(status), timeout_ns,
                                     cur_stream());
             },
             "Launches a one-thread kernel that polls the counter for 1..steps (bounded).");

    py::class_<Context>(p, "Context")
        .def(py::init<SymmetricHeap&, size_t, uint64_t>(), py::arg("heap"), py::arg("num_queues") = 1,
             py::arg("queue_capacity") = 2048, py::keep_alive<1, 2>())
        .def("spawn_proxy_threads", &Context::spawn_proxy_threads, py::arg("num_threads") = 1,
             py::arg("cpus") = std::vector<int>{})
        .def("join_proxy_threads", &Context::join_proxy_threads, py::call_guard<py::gil_scoped_release>())
        .def_property_readonly(
            "proxy_stats",
            [](const Context& c) {
                const auto st = c.proxy_stats();
                py::dict d;
                d["messages"] = st.callbacks;
                d["sweeps"] = st.sweeps;
                d["empty_polls"] = st.empty_polls;
                d["threads"] = st.threads;
                d["copies_issued"] = c.copies_issued();
                return d;
            },
            "Proxy totals: control messages served, sweeps, empty endpoint polls, threads, copy-engine puts.")
        .def_property_readonly("copies_issued", &Context::copies_issued)
        .def("set_active_queues", &Context::set_active_queues, py::arg("n"),
             "Proxy threads serve only control queues [0, n) (0 = all); returns the request's generation.")
        .def("active_applied", &Context::active_applied, py::arg("generation"))
        .def("ce_pingpong",
             [](Context& c, int peer, bool initiator, uint64_t bytes, uint32_t iters, uint32_t warmup,
                uint64_t src_off, uint64_t dst_off, uint64_t flag_off, torch::Tensor lat, torch::Tensor status,
                uint64_t timeout_ns) {
                 if (lat.numel() < iters) throw kiwi::error("ce_pingpong: lat needs iters entries");
                 launch_ce_pingpong(c.device_context(), peer, initiator, bytes, iters, warmup, src_off, dst_off,
                                    flag_off, u64_ptr(lat), u32_ptr(status), timeout_ns, cur_stream());
             })
        .def("ce_put_selftest",
             [](Context& c, int dst, uint64_t src_off, uint64_t dst_off, uint64_t bytes, uint32_t n,
                uint64_t flag_off, uint64_t counter_off, torch::Tensor status, uint64_t timeout_ns) {
                 launch_ce_put_selftest(c.device_context(), dst, src_off, dst_off, bytes, n, flag_off, counter_off,
                                        u32_ptr(status), timeout_ns, cur_stream());
             });

    py::class_<SymmetricHeap>(p, "SymmetricHeap")
        .def(py::init([](int device, size_t bytes, int rank, int world, const std::string& job, bool mc,
                         py::object barrier) {
                 SymmetricHeap::Barrier b;
                 if (!barrier.is_none()) {
                     auto fn = std::make_shared<py::object>(barrier);
                     b = [fn] {
                         py::gil_scoped_acquire g;
                         (*fn)();
                     };
                 }
                 py::gil_scoped_release nogil;
                 return new SymmetricHeap(device, bytes, rank, world, job, mc, b);
             }),
             py::arg("device"), py::arg("bytes"), py::arg("rank"), py::arg("world"), py::arg("job"),
             py::arg("multicast") = false, py::arg("barrier") = py::none())
        .def_property_readonly("size", &SymmetricHeap::size)
        .def_property_readonly("rank", &SymmetricHeap::rank)
        .def_property_readonly("world", &SymmetricHeap::world)
        .def_property_readonly("local_ptr", [](SymmetricHeap& h) { return reinterpret_cast<uintptr_t>(h.local()); })
        .def_property_readonly("mc_ptr", [](SymmetricHeap& h) { return reinterpret_cast<uintptr_t>(h.multicast()); })
        .def("peer_ptr", [](SymmetricHeap& h, int r) { return reinterpret_cast<uintptr_t>(h.peer(r)); })
        .def(
            "set_checks",
            [](SymmetricHeap& h, py::object record, uint64_t limit) {
                if (record.is_none()) {
                    h.set_checks(nullptr, 0);
                    return;
                }
                torch::Tensor t = record.cast<torch::Tensor>();
                TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kInt32 && t.numel() >= 4 && t.is_contiguous(),
                            "check record must be a contiguous int32 CUDA tensor of 4 words");
                h.set_checks(u32_ptr(t), limit);
            },
            py::arg("record"), py::arg("limit") = 0,
            "Checked mode of the device API: ranges validated against [0, limit) (0: the heap size), the first "
            "violation recorded in `record` as {1, site, rank, offset}, bad accesses skipped.  None: off.  Applies "
            "to views taken after the call.")
        .def_property_readonly("check_limit", [](SymmetricHeap& h) { return h.view().check_limit; })
        .def("checked_ops",
             [](SymmetricHeap& h, int peer, uint64_t off, uint64_t bytes, uint64_t flag_off) {
                 launch_checked_ops(h.view(), peer, off, bytes, flag_off, cur_stream());
             },
             py::arg("peer"), py::arg("off"), py::arg("bytes"), py::arg("flag_off"),
             "One block: put_block, get_block and signal on the given ranges (checked-mode tests).")
        .def("tensor",
             [](SymmetricHeap& h, uint64_t offset, std::vector<int64_t> shape, torch::Dtype dtype) {
                 int dev = 0;
                 cudaGetDevice(&dev);
                 return view_tensor(h.local(), h.size(), dev, offset, shape, dtype);
             },
             "View of this rank's heap memory (local only).")
        .def("pingpong",
             [](SymmetricHeap& h, int peer, bool initiator, uint64_t bytes, uint64_t iters, uint64_t warmup,
                uint64_t src_off, uint64_t dst_off, uint64_t flag_off, torch::Tensor lat, torch::Tensor status,
                uint32_t max_blocks, uint64_t timeout_ns) {
                 launch_pingpong(h.view(), peer, initiator, bytes, iters, warmup, src_off, dst_off, flag_off,
                                 u64_ptr(lat), u32_ptr(status), max_blocks, timeout_ns, cur_stream());
             })
        .def("pingpong_ll8",
             [](SymmetricHeap& h, int peer, bool initiator, uint32_t words, uint64_t iters, uint64_t warmup,
                uint64_t buf_off, torch::Tensor lat, torch::Tensor status, uint64_t timeout_ns) {
                 launch_pingpong_ll8(h.view(), peer, initiator, words, iters, warmup, buf_off, u64_ptr(lat),
                                     u32_ptr(status), timeout_ns, cur_stream());
             })
        .def("put_bw",
             [](SymmetricHeap& h, int peer, bool sender, uint64_t bytes, uint64_t reps, uint64_t src_off,
                uint64_t dst_off, uint64_t flag_off, uint64_t round, torch::Tensor elapsed, torch::Tensor status,
                uint32_t max_blocks, uint64_t timeout_ns, uint64_t region) {
                 launch_put_bw(h.view(), peer, sender, bytes, reps, src_off, dst_off, flag_off, round,
                               u64_ptr(elapsed), u32_ptr(status), max_blocks, timeout_ns, cur_stream(), region);
             },
             py::arg("peer"), py::arg("sender"), py::arg("bytes"), py::arg("reps"), py::arg("src_off"),
             py::arg("dst_off"), py::arg("flag_off"), py::arg("round"), py::arg("elapsed"), py::arg("status"),
             py::arg("max_blocks"), py::arg("timeout_ns"), py::arg("region") = 0)
        .def("get",
             [](SymmetricHeap& h, int peer, uint64_t bytes, uint64_t reps, uint64_t src_off, uint64_t dst_off,
                torch::Tensor lat, uint32_t max_blocks, uint64_t region) {
                 launch_get(h.view(), peer, bytes, reps, src_off, dst_off, u64_ptr(lat), max_blocks, cur_stream(),
                            region);
             },
             py::arg("peer"), py::arg("bytes"), py::arg("reps"), py::arg("src_off"), py::arg("dst_off"),
             py::arg("lat"), py::arg("max_blocks"), py::arg("region") = 0)
        .def("host_ce_pingpong", &host_ce_pingpong, py::arg("peer"), py::arg("initiator"), py::arg("bytes"),
             py::arg("iters"), py::arg("warmup"), py::arg("src_off"), py::arg("dst_off"), py::arg("flag_off"),
             py::arg("timeout_s") = 10.0, py::call_guard<py::gil_scoped_release>())
        .def("all2all_rounds",
             [](SymmetricHeap& h, uint64_t ingress_off, std::optional<torch::Tensor> send,
                std::optional<torch::Tensor> recv, torch::Tensor epoch, torch::Tensor status, uint64_t timeout_ns,
                uint32_t rounds, std::optional<torch::Tensor> lat) {
                 if (send.has_value() != recv.has_value()) throw kiwi::error("all2all_rounds: send and recv together");
                 if (send && (send->numel() < h.world() || recv->numel() < static_cast<int64_t>(rounds) * h.world())) {
                     throw kiwi::error("all2all_rounds: send needs world values, recv rounds x world");
                 }
                 if (lat && lat->numel() < static_cast<int64_t>(rounds)) throw kiwi::error("all2all_rounds: lat too small");
                 if (ingress_off + coll_ingress_bytes(h.world()) > h.size()) throw kiwi::error("all2all_rounds: ingress outside the heap");
                 launch_all2all_rounds(h.view(), ingress_off, send ? u32_ptr(*send) : nullptr,
                                       recv ? u32_ptr(*recv) : nullptr, u32_ptr(epoch), u32_ptr(status), timeout_ns,
                                       rounds, lat ? u64_ptr(*lat) : nullptr, cur_stream());
             },
             py::arg("ingress_off"), py::arg("send"), py::arg("recv"), py::arg("epoch"), py::arg("status"),
             py::arg("timeout_ns"), py::arg("rounds") = 1, py::arg("lat") = py::none())
        .def("coll_wait_only",
             [](SymmetricHeap& h, uint64_t ingress_off, uint32_t epoch, int src, torch::Tensor status,
                uint64_t timeout_ns, torch::Tensor waited) {
                 launch_coll_wait_only(h.view(), ingress_off, epoch, src, u32_ptr(status), timeout_ns, u64_ptr(waited),
                                       cur_stream());
             })
        .def("all_pairs",
             [](SymmetricHeap& h, uint64_t data_off, uint64_t flag_off, uint64_t words, uint32_t round,
                torch::Tensor status, uint64_t timeout_ns) {
                 launch_all_pairs(h.view(), data_off, flag_off, words, round, u32_ptr(status), timeout_ns,
                                  cur_stream());
             })
        .def("mc_broadcast",
             [](SymmetricHeap& h, int root, uint64_t src_off, uint64_t dst_off, uint64_t bytes, uint64_t flag_off) {
                 launch_mc_broadcast(h.view(), root, src_off, dst_off, bytes, flag_off, cur_stream());
             })
        .def("mc_allreduce_f32",
             [](SymmetricHeap& h, uint64_t off, uint64_t count) {
                 launch_mc_allreduce_f32(h.view(), off, count, cur_stream());
             })
        .def("wait_flag",
             [](SymmetricHeap& h, uint64_t flag_off, uint64_t want, torch::Tensor status, uint64_t timeout_ns) {
                 launch_wait_flag(h.view(), flag_off, want, u32_ptr(status), timeout_ns, cur_stream());
             })
        .def("barrier",
             [](SymmetricHeap& h, uint64_t flag_off, uint64_t round, torch::Tensor status, uint64_t timeout_ns) {
                 launch_heap_barrier(h.view(), flag_off, round, u32_ptr(status), timeout_ns, cur_stream());
             });
}
