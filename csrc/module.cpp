// Python bindings: kiwi_b200._C
//
// Sub-modules:  queue, invoke, bench, topology, p2p, ep.
// Parity: the reference exposes its core to Python only through Triton/FlyDSL
// byte-layout mirrors (python/kiwi_triton.py:36-47 of AMDResearch/kiwi) and a
// pybind EP op (apps/ep/python/kiwi_ep_bindings.hip.cpp).  Here the C++ core
// itself is bound, so Python code (and PyTorch extensions built against the
// headers) drive the same Context, queues and kernels.
#include <pybind11/functional.h>
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <memory>
#include <optional>

#include "kiwi/bench/gpu_bench.hpp"
#include "kiwi/bench/host_bench.hpp"
#include "kiwi/invoke/invoke.hpp"
#include "kiwi/invoke/printer.hpp"
#include "kiwi/invoke/progress.hpp"
#include "kiwi/topology.hpp"

namespace py = pybind11;
using namespace kiwi;

void register_p2p(py::module_& m);
void register_ep(py::module_& m);
void register_ops(py::module_& m);

namespace {

template <typename T>
py::array_t<T> to_numpy(const std::vector<T>& v) {
    py::array_t<T> a(v.size());
    if (!v.empty()) std::memcpy(a.mutable_data(), v.data(), v.size() * sizeof(T));
    return a;
}

/// A Python callable kept alive by C++; released with the GIL held.
struct PyFn {
    std::shared_ptr<py::object> fn;
    explicit PyFn(py::object f)
        : fn(new py::object(std::move(f)), [](py::object* p) {
              py::gil_scoped_acquire g;
              delete p;
          }) {}
    void operator()(const uint8_t* args, uint32_t bytes) const {
        py::gil_scoped_acquire g;
        (*fn)(py::bytes(reinterpret_cast<const char*>(args), bytes));
    }
};

/// Type-erased invoke::Context for Python (SPSC or MPSC endpoints).
class KiwiContextBase {
public:
    virtual ~KiwiContextBase() = default;
    virtual uint8_t register_callback(py::object fn, int64_t nbytes) = 0;
    virtual size_t progress(size_t ep, int max) = 0;
    virtual size_t progress_all(int max) = 0;
    virtual void start_threads(size_t n, std::vector<int> cpus) = 0;
    virtual void stop_threads() = 0;
    virtual uint32_t set_active_endpoints(size_t n) = 0;
    virtual size_t active_endpoints() const = 0;
    virtual bool active_applied(uint32_t generation) const = 0;
    virtual uint64_t callbacks_run() const = 0;
    virtual invoke::ProgressStats stats() const = 0;
    virtual uintptr_t device_context_ptr() const = 0;
    virtual size_t num_endpoints() const = 0;
    virtual size_t num_callbacks() const = 0;
    virtual void emulate_invoke(size_t ep, uint8_t cb, py::bytes payload) = 0;
    virtual void check_device_errors() = 0;
    virtual void rethrow() = 0;
    virtual bool poll_ready(size_t ep) = 0;
    virtual void upload_handles() = 0;
    virtual bool host_only() const = 0;
    /// A native callback (any payload) that only counts its calls: lets a
    /// benchmark measure the queue / frontend without Python in the loop.
    virtual uint8_t register_native_counter() = 0;
    /// A native callback taking one uint32 n that sets the progress threads'
    /// active prefix (0 = all): how a kernel publishes the endpoints it uses.
    virtual uint8_t register_active_endpoints_callback() = 0;
    virtual uint64_t native_count() const = 0;
    /// A native callback that prints its arguments with a printf-style format.
    virtual uint8_t register_native_print(const std::string& fmt, const std::string& codes, bool to_stderr) = 0;
};

template <typename Q>
class KiwiContext final : public KiwiContextBase {
public:
    KiwiContext(size_t n, uint64_t cap, bool host_only)
        : ctx_(n, cap, host_only ? queue::MemKind::kHost : queue::default_host_kind()),
          threads_(ctx_), host_only_(host_only || ctx_.memory_kind() == queue::MemKind::kHost) {}
    ~KiwiContext() override {
        py::gil_scoped_release nogil;
        threads_.stop();
    }
    uint8_t register_callback(py::object fn, int64_t nbytes) override {
        const uint32_t exp = nbytes < 0 ? invoke::CallbackBase::kAnySize : static_cast<uint32_t>(nbytes);
        return ctx_.register_raw_callback(PyFn(std::move(fn)), exp);
    }
    uint8_t register_native_counter() override {
        return ctx_.register_raw_callback(
            [this](const uint8_t*, uint32_t) { count_.fetch_add(1, std::memory_order_relaxed); },
            invoke::CallbackBase::kAnySize);
    }
    uint8_t register_active_endpoints_callback() override {
        return ctx_.register_callback(
            std::function<void(uint32_t)>([this](uint32_t n) { threads_.set_active_endpoints(n); }));
    }
    uint64_t native_count() const override { return count_.load(std::memory_order_relaxed); }
    uint8_t register_native_print(const std::string& fmt, const std::string& codes, bool to_stderr) override {
        invoke::PrintFormat pf(fmt, codes);  // throws on a bad format, at registration
        const uint32_t bytes = pf.payload_bytes();
        return ctx_.register_raw_callback(
            [pf, to_stderr](const uint8_t* p, uint32_t n) { pf.print(p, n, to_stderr ? stderr : stdout); }, bytes);
    }
    size_t progress(size_t ep, int max) override { return ctx_.progress(ep, max); }
    size_t progress_all(int max) override { return ctx_.progress_all(max); }
    void start_threads(size_t n, std::vector<int> cpus) override { threads_.start(n, std::move(cpus)); }
    void stop_threads() override {
        py::gil_scoped_release nogil;
        threads_.stop();
    }
    uint32_t set_active_endpoints(size_t n) override { return threads_.set_active_endpoints(n); }
    size_t active_endpoints() const override { return threads_.active_endpoints(); }
    bool active_applied(uint32_t generation) const override { return threads_.active_applied(generation); }
    uint64_t callbacks_run() const override { return threads_.callbacks_run(); }
    invoke::ProgressStats stats() const override { return threads_.stats(); }
    uintptr_t device_context_ptr() const override {
        return reinterpret_cast<uintptr_t>(ctx_.device_context());
    }
    size_t num_endpoints() const override { return ctx_.num_endpoints(); }
    size_t num_callbacks() const override { return ctx_.num_callbacks(); }
    void emulate_invoke(size_t ep, uint8_t cb, py::bytes payload) override {
        if (!host_only_) throw kiwi::error("emulate_invoke needs a host-only context");
        auto it = writers_.find(ep);
        if (it == writers_.end()) {
            it = writers_.emplace(ep, ctx_.raw_queue(ep)->host_writer_any()).first;
        }
        std::string s = payload;
        while (!it->second.try_push(s.data(), static_cast<uint32_t>(s.size()), cb)) {
            throw kiwi::error("emulate_invoke: ring full (call progress first)");
        }
    }
    void check_device_errors() override { ctx_.check_device_errors(); }
    void rethrow() override { threads_.rethrow_if_failed(); }
    bool poll_ready(size_t ep) override { return ctx_.poll_state(ep).ready(); }
    void upload_handles() override { ctx_.upload_handles(); }
    bool host_only() const override { return host_only_; }

private:
    std::atomic<uint64_t> count_{0};
    invoke::Context<Q> ctx_;
    invoke::ProgressThreads<Q> threads_;
    bool host_only_;
    std::map<size_t, queue::RingWriter> writers_;
};

}  // namespace

PYBIND11_MODULE(_C, m) {
    m.doc() = "kiwi_b200 native core";
    m.attr("version") = py::make_tuple(KIWI_VERSION_MAJOR, KIWI_VERSION_MINOR, KIWI_VERSION_PATCH);
    m.def("cuda_device_available", &queue::cuda_device_available);

    // ---------------- queue ----------------
    auto q = m.def_submodule("queue", "kiwi::queue rings");
    q.attr("MAX_MESSAGE_BYTES") = queue::kMaxMessageBytes;
    q.attr("LINE_BYTES") = queue::kLineBytes;
    q.attr("CHUNK_BYTES") = queue::kChunkBytes;
    q.attr("MAX_CAPACITY_LINES") = queue::kMaxCapacityLines;
    q.def("message_lines", [](uint32_t b) { return queue::message_lines(b); });
    q.def("message_chunks", [](uint32_t b) { return queue::message_chunks(b); });
    q.def("lap_tag", [](uint64_t line, uint64_t cap) { return queue::lap_tag(line, log2_pow2(cap)); });
    q.def("handle_layout", [] {
        py::dict d;
        d["SpscD2HHandle"] = sizeof(queue::SpscD2HHandle);
        d["MpscD2HHandle"] = sizeof(queue::MpscD2HHandle);
        d["SpscH2DHandle"] = sizeof(queue::SpscH2DHandle);
        d["MpmcH2DHandle"] = sizeof(queue::MpmcH2DHandle);
        d["SpscD2HHandle.ring"] = offsetof(queue::SpscD2HHandle, ring);
        d["SpscD2HHandle.consumer_pos"] = offsetof(queue::SpscD2HHandle, consumer_pos);
        d["SpscD2HHandle.err"] = offsetof(queue::SpscD2HHandle, err);
        d["SpscD2HHandle.head"] = offsetof(queue::SpscD2HHandle, head);
        d["SpscD2HHandle.credit_limit"] = offsetof(queue::SpscD2HHandle, credit_limit);
        d["SpscD2HHandle.log2cap"] = offsetof(queue::SpscD2HHandle, log2cap);
        d["InvokeHandle<SPSC>"] = sizeof(invoke::InvokeHandle<queue::SpscD2HHandle>);
        d["DeviceContext<SPSC>"] = sizeof(invoke::DeviceContext<queue::SPSCD2HQueue>);
        d["ErrorRecord"] = sizeof(ErrorRecord);
        return d;
    });

    py::class_<queue::HostPollState>(q, "HostPollState")
        .def("ready", &queue::HostPollState::ready)
        .def("refresh", &queue::HostPollState::refresh);

    py::class_<queue::RingWriter>(q, "RingWriter")
        .def("try_push",
             [](queue::RingWriter& w, py::bytes payload, uint32_t meta) {
                 std::string s = payload;
                 return w.try_push(s.data(), static_cast<uint32_t>(s.size()), meta);
             },
             py::arg("payload"), py::arg("metadata") = 0)
        .def("write_chunks",
             [](queue::RingWriter& w, py::bytes payload, uint32_t meta, uint32_t first, uint32_t last) {
                 std::string s = payload;
                 w.write_chunks(s.data(), static_cast<uint32_t>(s.size()), meta, first, last);
             },
             "Write chunks [first, last) of a message without advancing (fault injection).")
        .def("advance", &queue::RingWriter::advance)
        .def("lines_for", &queue::RingWriter::lines_for)
        .def_property_readonly("head", &queue::RingWriter::head);

    auto pop_to_py = [](queue::D2HRingBase& r) -> py::object {
        alignas(64) uint8_t buf[queue::kMaxMessageBytes];
        uint32_t meta = 0, bytes = 0;
        if (!r.try_pop(buf, &meta, &bytes)) return py::none();
        return py::make_tuple(py::bytes(reinterpret_cast<const char*>(buf), bytes), meta);
    };

    py::class_<queue::D2HRingBase>(q, "D2HRing")
        .def("try_pop", pop_to_py, "Pop one message -> (payload: bytes, metadata: int) or None")
        .def("host_poll_state", &queue::D2HRingBase::host_poll_state)
        .def_property_readonly("capacity", &queue::D2HRingBase::capacity)
        .def_property_readonly("consumer_position", &queue::D2HRingBase::consumer_position)
        .def("error", [](queue::D2HRingBase& r) {
            const auto e = r.error();
            return py::make_tuple(e.code, e.site, e.rank, e.info);
        })
        .def("corrupt_line", [](queue::D2HRingBase& r, uint64_t line, uint32_t chunk, uint32_t lo, uint32_t tag0,
                                uint32_t hi, uint32_t tag1) {
            queue::Chunk* c = &r.ring_host()[(line & (r.capacity() - 1)) * queue::kChunksPerLine + chunk];
            queue::host::store_half(&c->lo, queue::pack_half(lo, tag0));
            queue::host::store_half(&c->hi, queue::pack_half(hi, tag1));
        }, "Overwrite one chunk (fault injection on host-only rings).");

    py::class_<queue::SPSCD2HQueue, queue::D2HRingBase>(q, "SPSCD2HQueue")
        .def(py::init([](uint64_t cap, bool host_only) {
                 return new queue::SPSCD2HQueue(cap, host_only ? queue::MemKind::kHost : queue::default_host_kind());
             }),
             py::arg("capacity"), py::arg("host_only") = false)
        .def("host_writer", &queue::SPSCD2HQueue::host_writer,
             "CPU stand-in for the producer warp, positioned at the consumer.");

    py::class_<queue::MPSCD2HQueue, queue::D2HRingBase>(q, "MPSCD2HQueue")
        .def(py::init([](uint64_t cap, bool host_only) {
                 return new queue::MPSCD2HQueue(cap, host_only ? queue::MemKind::kHost : queue::default_host_kind());
             }),
             py::arg("capacity"), py::arg("host_only") = false)
        .def("host_writer", &queue::MPSCD2HQueue::host_writer_any);

    py::class_<queue::SPSCH2DQueue>(q, "SPSCH2DQueue")
        .def(py::init([](uint64_t cap, bool host_only, uint32_t notify) {
                 return new queue::SPSCH2DQueue(cap, host_only ? queue::MemKind::kHost : queue::default_host_kind(),
                                                notify);
             }),
             py::arg("capacity"), py::arg("host_only") = false, py::arg("notify_interval") = 1)
        .def("try_push",
             [](queue::SPSCH2DQueue& s, py::bytes payload, uint32_t meta) {
                 std::string b = payload;
                 return s.try_push(b.data(), static_cast<uint32_t>(b.size()), meta);
             },
             py::arg("payload"), py::arg("metadata") = 0)
        .def("host_reader", [](queue::SPSCH2DQueue& s) {
            // CPU stand-in for the consumer warp (host-only rings).
            return std::make_unique<queue::RingReader>(s.ring_host(), s.capacity(), s.consumer_pos_host(),
                                                       s.consumer_position());
        })
        .def_property_readonly("capacity", &queue::SPSCH2DQueue::capacity)
        .def_property_readonly("producer_position", &queue::SPSCH2DQueue::producer_position)
        .def_property_readonly("consumer_position", &queue::SPSCH2DQueue::consumer_position);

    py::class_<queue::RingReader>(q, "RingReader")
        .def("try_pop", [](queue::RingReader& r) -> py::object {
            alignas(64) uint8_t buf[queue::kMaxMessageBytes];
            uint32_t meta = 0, bytes = 0;
            if (!r.try_pop(buf, &meta, &bytes)) return py::none();
            return py::make_tuple(py::bytes(reinterpret_cast<const char*>(buf), bytes), meta);
        })
        .def_property_readonly("tail", &queue::RingReader::tail);

    py::class_<queue::MPMCH2DQueue>(q, "MPMCH2DQueue")
        .def(py::init([](uint64_t slots, uint32_t slot_lines, bool host_only) {
                 return new queue::MPMCH2DQueue(slots, slot_lines,
                                                host_only ? queue::MemKind::kHost : queue::default_host_kind());
             }),
             py::arg("slots"), py::arg("slot_lines") = 2, py::arg("host_only") = false)
        .def("try_push",
             [](queue::MPMCH2DQueue& s, py::bytes payload, uint32_t meta) {
                 std::string b = payload;
                 return s.try_push(b.data(), static_cast<uint32_t>(b.size()), meta);
             },
             py::arg("payload"), py::arg("metadata") = 0)
        .def(
            "host_try_pop",
            [](queue::MPMCH2DQueue& s) -> py::object {
                uint8_t buf[queue::kMaxMessageBytes];
                uint32_t meta = 0, bytes = 0;
                if (!s.host_try_pop(buf, &meta, &bytes)) return py::none();
                return py::make_tuple(py::bytes(reinterpret_cast<const char*>(buf), bytes), meta);
            },
            "CPU stand-in for the device consumers (host_only queues): (payload, metadata) or None.")
        .def_property_readonly("slot_payload_bytes", &queue::MPMCH2DQueue::slot_payload_bytes)
        .def_property_readonly("producer_position", &queue::MPMCH2DQueue::producer_position);

    // ---------------- invoke ----------------
    auto inv = m.def_submodule("invoke", "kiwi::invoke contexts");
    inv.attr("MAX_CALLBACKS") = invoke::kMaxCallbacks;
    py::class_<KiwiContextBase>(inv, "Context")
        .def(py::init([](size_t n, uint64_t cap, bool mpsc, bool host_only) -> KiwiContextBase* {
                 if (mpsc) return new KiwiContext<queue::MPSCD2HQueue>(n, cap, host_only);
                 return new KiwiContext<queue::SPSCD2HQueue>(n, cap, host_only);
             }),
             py::arg("num_endpoints") = 1, py::arg("capacity") = 4096, py::arg("mpsc") = false,
             py::arg("host_only") = false)
        .def("register_callback", &KiwiContextBase::register_callback, py::arg("fn"), py::arg("nbytes") = -1,
             "Register fn(payload: bytes); nbytes = exact payload size or -1 for any.")
        .def("progress", &KiwiContextBase::progress, py::arg("endpoint") = 0, py::arg("max_callbacks") = -1)
        .def("progress_all", &KiwiContextBase::progress_all, py::arg("max_per_endpoint") = -1)
        .def("start_progress_threads", &KiwiContextBase::start_threads, py::arg("num_threads") = 1,
             py::arg("cpus") = std::vector<int>{})
        .def("stop_progress_threads", &KiwiContextBase::stop_threads)
        .def("set_active_endpoints", &KiwiContextBase::set_active_endpoints, py::arg("n"),
             "Progress threads poll endpoints [0, n) only (0 = all); a shrink drains the dropped endpoints once. "
             "Returns the request's generation.")
        .def_property_readonly("active_endpoints", &KiwiContextBase::active_endpoints)
        .def("active_applied", &KiwiContextBase::active_applied, py::arg("generation"))
        .def_property_readonly("callbacks_run", &KiwiContextBase::callbacks_run)
        .def_property_readonly(
            "stats",
            [](const KiwiContextBase& c) {
                const auto st = c.stats();
                py::dict d;
                d["callbacks"] = st.callbacks;
                d["sweeps"] = st.sweeps;
                d["empty_polls"] = st.empty_polls;
                d["threads"] = st.threads;
                return d;
            },
            "Progress-thread totals: callbacks, sweeps, endpoint polls that found nothing, threads running.")
        .def_property_readonly("device_context_ptr", &KiwiContextBase::device_context_ptr)
        .def_property_readonly("num_endpoints", &KiwiContextBase::num_endpoints)
        .def_property_readonly("num_callbacks", &KiwiContextBase::num_callbacks)
        .def_property_readonly("host_only", &KiwiContextBase::host_only)
        .def("emulate_invoke", &KiwiContextBase::emulate_invoke,
             "Host-only contexts: push a message as the device would (tests).")
        .def("poll_ready", &KiwiContextBase::poll_ready)
        .def("upload_handles", &KiwiContextBase::upload_handles)
        .def("check_device_errors", &KiwiContextBase::check_device_errors)
        .def("rethrow_progress_errors", &KiwiContextBase::rethrow)
        .def("register_native_counter", &KiwiContextBase::register_native_counter)
        .def("register_active_endpoints_callback", &KiwiContextBase::register_active_endpoints_callback,
             "Registers a callback (one uint32 argument) that sets the active endpoint prefix; returns its id.")
        .def("register_native_print", &KiwiContextBase::register_native_print, py::arg("fmt"), py::arg("codes"),
             py::arg("to_stderr") = false,
             "Native callback printing its packed arguments (struct codes b B h H i I l L q Q f d) with a "
             "printf-style format; the format is checked against the codes here.")
        .def_property_readonly("native_count", &KiwiContextBase::native_count);

    m.def_submodule("print_format").def(
        "format",
        [](const std::string& fmt, const std::string& codes, py::bytes payload) {
            invoke::PrintFormat pf(fmt, codes);
            const std::string b = payload;
            return pf.format(reinterpret_cast<const uint8_t*>(b.data()), static_cast<uint32_t>(b.size()));
        },
        py::arg("fmt"), py::arg("codes"), py::arg("payload"),
        "What register_native_print would print for one payload (no newline).");

    // ---------------- bench ----------------
    auto b = m.def_submodule("bench", "native benchmark loops");
    b.def("host_ring_pingpong",
          [](uint64_t iters, uint64_t warmup, uint64_t cap, uint32_t bytes, uint64_t seed, int a, int c) {
              bench::HostRingResult r;
              {
                  py::gil_scoped_release nogil;
                  r = bench::host_ring_pingpong(iters, warmup, cap, bytes, seed, a, c);
              }
              py::dict d;
              d["latencies_ns"] = to_numpy(r.latencies_ns);
              d["total_ns"] = r.total_ns;
              d["checksum"] = r.checksum;
              d["ok"] = r.ok;
              return d;
          },
          py::arg("iters"), py::arg("warmup"), py::arg("capacity") = 4096, py::arg("payload_bytes") = 8,
          py::arg("seed") = 0, py::arg("cpu_a") = -1, py::arg("cpu_b") = -1);
    b.def("queue_baselines",
          [](uint64_t iters, uint64_t warmup, uint64_t messages, uint32_t bytes, uint64_t cap, int a, int c,
             uint64_t idle_polls, bool loaded, int cpu_c, int cpu_d) {
              bench::BaselineOptions o;
              o.iters = iters;
              o.warmup = warmup;
              o.messages = messages;
              o.payload_bytes = bytes;
              o.capacity = cap;
              o.cpu_a = a;
              o.cpu_b = c;
              o.idle_polls = idle_polls;
              o.loaded = loaded;
              o.cpu_c = cpu_c;
              o.cpu_d = cpu_d;
              std::vector<bench::BaselineResult> rs;
              {
                  py::gil_scoped_release nogil;
                  rs = bench::queue_baselines(o);
              }
              py::list out;
              for (const auto& r : rs) {
                  py::dict d;
                  d["name"] = r.name;
                  d["p50_ns"] = r.p50_ns;
                  d["p99_ns"] = r.p99_ns;
                  d["msgs_per_s"] = r.msgs_per_s;
                  if (idle_polls) d["idle_poll_ns"] = r.idle_poll_ns;
                  if (loaded) {
                      d["loaded_p50_ns"] = r.loaded_p50_ns;
                      d["loaded_p99_ns"] = r.loaded_p99_ns;
                      d["loaded_bg_msgs_per_s"] = r.loaded_bg_msgs_per_s;
                  }
                  d["ok"] = r.ok;
                  out.append(d);
              }
              return out;
          },
          py::arg("iters") = 100000, py::arg("warmup") = 10000, py::arg("messages") = 1000000,
          py::arg("payload_bytes") = 8, py::arg("capacity") = 4096, py::arg("cpu_a") = -1, py::arg("cpu_b") = -1,
          py::arg("idle_polls") = 0, py::arg("loaded") = false, py::arg("cpu_c") = -1, py::arg("cpu_d") = -1,
          "Host-only queue baselines (kiwi ring, head/tail ring, per-slot sequence ring, raw word): ping-pong, "
          "stream, and optionally the idle-poll cost and the loaded ping-pong.");
    b.def("gpu_queue_baseline",
          [](const std::string& queue, const std::string& mode, uint64_t iters, uint64_t warmup, uint32_t warps,
             uint64_t capacity, int cpu, uint64_t timeout_ns) {
              bench::GpuQueueBaselineOptions o;
              o.queue = queue;
              o.mode = mode;
              o.iters = iters;
              o.warmup = warmup;
              o.warps = warps;
              o.capacity = capacity;
              o.cpu = cpu;
              o.timeout_ns = timeout_ns;
              bench::GpuQueueBaselineResult r;
              {
                  py::gil_scoped_release nogil;
                  r = bench::gpu_queue_baseline(o);
              }
              py::dict d;
              d["queue"] = r.queue;
              d["mode"] = r.mode;
              d["ok"] = r.ok;
              d["status"] = r.status;
              d["messages"] = r.messages;
              d["bad"] = r.bad;
              d["order_errors"] = r.order_errors;
              d["seconds"] = r.seconds;
              d["cycles_per_push"] = r.cycles_per_push;
              d["lat_ns"] = to_numpy(r.lat_ns);
              return d;
          },
          py::arg("queue"), py::arg("mode") = "latency", py::arg("iters") = 10000, py::arg("warmup") = 1000,
          py::arg("warps") = 1, py::arg("capacity") = 4096, py::arg("cpu") = -1,
          py::arg("timeout_ns") = 2000000000ull,
          "GPU-producer queue comparators (kiwi_spsc, kiwi_mpsc, fifo_trigger, proxy_channel, raw_store) in latency, "
          "throughput or push_cost mode; a pinned host thread consumes and validates every message.");
    b.def("host_ring_stream",
          [](uint64_t n, uint64_t cap, uint32_t bytes, uint64_t seed, int a, int c) {
              bench::HostRingResult r;
              {
                  py::gil_scoped_release nogil;
                  r = bench::host_ring_stream(n, cap, bytes, seed, a, c);
              }
              py::dict d;
              d["total_ns"] = r.total_ns;
              d["checksum"] = r.checksum;
              d["ok"] = r.ok;
              return d;
          },
          py::arg("messages"), py::arg("capacity") = 4096, py::arg("payload_bytes") = 8, py::arg("seed") = 0,
          py::arg("cpu_a") = -1, py::arg("cpu_b") = -1);
    b.def("xorshift64", [](uint64_t s) { return bench::xorshift64(s); });

    auto rtt_to_dict = [](const bench::RttResult& r) {
        py::dict d;
        d["lat_ns"] = to_numpy(r.lat_ns);
        d["lat_cycles"] = to_numpy(r.lat_cycles);
        d["total_ns"] = r.total_ns;
        d["total_cycles"] = r.total_cycles;
        d["callbacks"] = r.callbacks;
        d["status"] = r.status;
        d["ok"] = r.ok;
        return d;
    };
    b.def("invoke_rtt",
          [rtt_to_dict](uint64_t iters, uint64_t warmup, uint32_t bytes, uint64_t seed, int cpu, uint64_t cap,
                        bool mpsc, uint32_t poll_warps, uint64_t timeout_ns, bool mailbox, uint32_t stagger_ns,
                        uint32_t initial_delay_ns, uint32_t pipeline, bool adaptive, bool demote,
                        uint32_t block_threads) {
              bench::RttConfig c;
              c.iters = iters;
              c.warmup = warmup;
              c.payload_bytes = bytes;
              c.seed = seed;
              c.cpu = cpu;
              c.capacity = cap;
              c.mpsc = mpsc;
              c.poll_warps = poll_warps;
              c.timeout_ns = timeout_ns;
              c.mailbox = mailbox;
              c.stagger_ns = stagger_ns;
              c.initial_delay_ns = initial_delay_ns;
              c.pipeline = pipeline;
              c.adaptive = adaptive;
              c.demote = demote;
              c.block_threads = block_threads;
              bench::RttResult r;
              {
                  py::gil_scoped_release nogil;
                  r = bench::invoke_rtt(c);
              }
              return rtt_to_dict(r);
          },
          py::arg("iters") = 100000, py::arg("warmup") = 10000, py::arg("payload_bytes") = 8, py::arg("seed") = 1,
          py::arg("cpu") = -1, py::arg("capacity") = 4096, py::arg("mpsc") = false, py::arg("poll_warps") = 0,
          py::arg("timeout_ns") = 2000000000ull, py::arg("mailbox") = false, py::arg("stagger_ns") = 200,
          py::arg("initial_delay_ns") = 300, py::arg("pipeline") = 1, py::arg("adaptive") = true,
          py::arg("demote") = true, py::arg("block_threads") = 0);
    b.def("pcie_floor",
          [rtt_to_dict](uint64_t iters, uint64_t warmup, int cpu, uint64_t timeout_ns) {
              bench::RttResult r;
              {
                  py::gil_scoped_release nogil;
                  r = bench::pcie_floor(iters, warmup, cpu, timeout_ns);
              }
              return rtt_to_dict(r);
          },
          py::arg("iters") = 100000, py::arg("warmup") = 10000, py::arg("cpu") = -1,
          py::arg("timeout_ns") = 2000000000ull);

    b.def("rtt_lab",
          [rtt_to_dict](uint64_t iters, uint64_t warmup, uint32_t pollers, uint32_t mirrors, uint32_t stagger,
                        uint32_t fence, uint32_t pipeline, int cpu, uint32_t delay) {
              bench::RttResult r;
              {
                  py::gil_scoped_release nogil;
                  r = bench::rtt_lab(iters, warmup, pollers, mirrors, stagger, fence, pipeline, cpu, delay);
              }
              return rtt_to_dict(r);
          },
          py::arg("iters") = 100000, py::arg("warmup") = 10000, py::arg("pollers") = 0, py::arg("mirrors") = 1,
          py::arg("stagger_ns") = 0, py::arg("fence") = 0, py::arg("pipeline") = 1, py::arg("cpu") = -1,
          py::arg("initial_delay_ns") = 0);

    auto push_to_dict = [](const bench::PushTestResult& r) {
        py::dict d;
        d["popped"] = r.popped;
        d["mismatches"] = r.mismatches;
        d["order_errors"] = r.order_errors;
        d["device_error"] = r.device_error;
        d["first_error"] = r.first_error;
        return d;
    };
    b.def("d2h_push_test",
          [push_to_dict](const std::string& mode, bool mpsc, uint64_t cap, uint32_t warps, uint32_t msgs,
                         std::vector<uint32_t> sizes, uint32_t launches, uint64_t seed) {
              bench::PushTestResult r;
              {
                  py::gil_scoped_release nogil;
                  r = bench::d2h_push_test(mode, mpsc, cap, warps, msgs, sizes, launches, seed);
              }
              return push_to_dict(r);
          },
          py::arg("mode"), py::arg("mpsc") = false, py::arg("capacity") = 64, py::arg("warps") = 1,
          py::arg("msgs_per_warp") = 100, py::arg("sizes") = std::vector<uint32_t>{8}, py::arg("launches") = 1,
          py::arg("seed") = 7);
    b.def("h2d_spsc_test",
          [push_to_dict](uint64_t cap, uint32_t count, std::vector<uint32_t> sizes, bool regs, uint32_t notify,
                         uint64_t seed) {
              bench::PushTestResult r;
              {
                  py::gil_scoped_release nogil;
                  r = bench::h2d_spsc_test(cap, count, sizes, regs, notify, seed);
              }
              return push_to_dict(r);
          },
          py::arg("capacity") = 16, py::arg("count") = 100, py::arg("sizes") = std::vector<uint32_t>{8},
          py::arg("registers") = true, py::arg("notify_interval") = 1, py::arg("seed") = 3);
    b.def("h2d_mpmc_test",
          [push_to_dict](uint64_t slots, uint32_t slot_lines, uint32_t producers, uint32_t msgs, uint32_t warps,
                         uint64_t seed) {
              bench::PushTestResult r;
              {
                  py::gil_scoped_release nogil;
                  r = bench::h2d_mpmc_test(slots, slot_lines, producers, msgs, warps, seed);
              }
              return push_to_dict(r);
          },
          py::arg("slots") = 16, py::arg("slot_lines") = 2, py::arg("producers") = 2,
          py::arg("msgs_per_producer") = 100, py::arg("warps") = 4, py::arg("seed") = 5);
    b.def("atomicity_test", [](uint32_t iters, uint32_t mode) {
        bench::AtomicityResult r;
        {
            py::gil_scoped_release nogil;
            r = bench::atomicity_test(iters, mode);
        }
        py::dict d;
        d["reads"] = r.reads;
        d["torn8"] = r.torn8;
        d["tag_ahead"] = r.tag_ahead;
        d["split16"] = r.split16;
        d["torn_word"] = r.torn_word;
        d["torn_nonzero"] = r.torn_nonzero;
        d["final_ok"] = r.final_ok;
        d["samples"] = r.samples;
        return d;
    }, py::arg("iters"), py::arg("mode") = 0);
    b.def("atomicity_protocol_test", [](uint32_t iters, uint32_t format) {
        bench::ProtocolResult r;
        {
            py::gil_scoped_release nogil;
            r = bench::atomicity_protocol_test(iters, format);
        }
        py::dict d;
        d["rounds"] = r.rounds;
        d["reads"] = r.reads;
        d["torn"] = r.torn;
        d["accepted_bad"] = r.accepted_bad;
        d["ok"] = r.ok;
        d["samples"] = r.samples;
        return d;
    }, py::arg("iters"), py::arg("format") = 0);
    b.def("atomicity_h2d_test", [](uint32_t duration_ms) {
        bench::AtomicityResult r;
        {
            py::gil_scoped_release nogil;
            r = bench::atomicity_h2d_test(duration_ms);
        }
        py::dict d;
        d["reads"] = r.reads;
        d["torn8"] = r.torn8;
        d["split16"] = r.split16;
        d["torn_word"] = r.torn_word;
        d["torn_nonzero"] = r.torn_nonzero;
        d["final_ok"] = r.final_ok;
        d["samples"] = r.samples;
        return d;
    }, py::arg("duration_ms"));
    b.def("invoke_throughput",
          [](uint32_t endpoints, uint32_t threads, uint32_t msgs, uint32_t bytes, uint64_t cap) {
              bench::ThroughputResult r;
              {
                  py::gil_scoped_release nogil;
                  r = bench::invoke_throughput(endpoints, threads, msgs, bytes, cap);
              }
              py::dict d;
              d["messages"] = r.messages;
              d["device_ns"] = r.device_ns;
              d["ok"] = r.ok;
              return d;
          },
          py::arg("endpoints") = 4, py::arg("threads") = 1, py::arg("msgs_per_endpoint") = 10000,
          py::arg("payload_bytes") = 8, py::arg("capacity") = 4096);
    b.def("push_cost",
          [](uint32_t msgs, uint32_t bytes) {
              bench::PushCostResult r;
              {
                  py::gil_scoped_release nogil;
                  r = bench::push_cost(msgs, bytes);
              }
              py::dict d;
              d["cycles_per_push"] = r.cycles_per_push;
              d["ok"] = r.ok;
              return d;
          },
          py::arg("msgs") = 10000, py::arg("payload_bytes") = 8);
    b.def("grid_poll",
          [](uint32_t blocks, uint32_t threads, uint32_t rounds, uint64_t delay_ns, uint64_t timeout_ns) {
              bench::GridPollResult r;
              {
                  py::gil_scoped_release nogil;
                  r = bench::grid_poll(blocks, threads, rounds, delay_ns, timeout_ns);
              }
              py::dict d;
              d["blocks"] = r.blocks;
              d["pollers"] = r.pollers;
              d["first_observe_p50_ns"] = r.first_observe_p50_ns;
              d["last_observe_p50_ns"] = r.last_observe_p50_ns;
              d["last_observe_p99_ns"] = r.last_observe_p99_ns;
              d["ack_p50_ns"] = r.ack_p50_ns;
              d["ack_p99_ns"] = r.ack_p99_ns;
              d["status"] = r.status;
              d["ok"] = r.ok;
              return d;
          },
          py::arg("blocks") = 16, py::arg("threads") = 256, py::arg("rounds") = 1000, py::arg("delay_ns") = 10000,
          py::arg("timeout_ns") = 2000000000ull,
          "Host-mapped grid polling: block 0 publishes, every other block's warps poll, blocks ack back.");
    b.def("invoke_cost",
          [](uint32_t calls, bool lane_masked) {
              bench::InvokeCostResult r;
              {
                  py::gil_scoped_release nogil;
                  r = bench::invoke_cost(calls, lane_masked);
              }
              py::dict d;
              d["cycles_per_call"] = r.cycles_per_call;
              d["messages"] = r.messages;
              d["ok"] = r.ok;
              return d;
          },
          py::arg("calls") = 10000, py::arg("lane_masked") = false,
          "SM cycles per device invoke (16-byte arguments), or per lane-masked invoke of 16 lanes.");
    b.def("h2d_timeout_test", [](uint64_t ns) {
        py::gil_scoped_release nogil;
        return bench::h2d_timeout_test(ns);
    });
    b.def("queue_kernel_attributes", [] {
        py::list out;
        for (const auto& a : bench::queue_kernel_attributes()) {
            out.append(py::make_tuple(a.name, a.local_bytes, a.registers));
        }
        return out;
    });

    // ---------------- topology ----------------
    auto t = m.def_submodule("topology", "CPU affinity helpers");
    t.def("pci_bus_id", &topology::pci_bus_id);
    t.def("parse_cpulist", &topology::parse_cpulist);
    t.def("gpu_local_cpus", &topology::gpu_local_cpus, py::arg("device"), py::arg("sysfs_root") = "/sys");
    t.def("process_cpus", &topology::process_cpus);
    t.def("poller_cpus", &topology::poller_cpus, py::arg("device"), py::arg("n"), py::arg("sysfs_root") = "/sys");
    t.def("bind_current_thread", &topology::bind_current_thread);
    t.def("current_thread_cpus", &topology::current_thread_cpus);
    t.def("gpu_numa_node", &topology::gpu_numa_node, py::arg("device"), py::arg("sysfs_root") = "/sys");

    register_p2p(m);
    register_ep(m);
    register_ops(m);
}
