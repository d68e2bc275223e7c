// Host progress threads for a kiwi::invoke::Context.
//
// Parity with the reference's proxy threads (apps/p2p/context.hip.cpp:212-311
// of AMDResearch/kiwi): thread t owns endpoints t, t+T, ...; a sweep checks
// each owned endpoint with its HostPollState (one load) and only then runs
// progress() and refreshes the state; an optional hook runs once per endpoint
// per sweep; threads are pinned to GPU-local CPUs; stop() drains.
#pragma once

#include <atomic>
#include <exception>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

#include "kiwi/invoke/invoke.hpp"
#include "kiwi/topology.hpp"

namespace kiwi::invoke {

template <typename Queue>
class ProgressThreads {
public:
    using Hook = std::function<void(size_t endpoint)>;

    explicit ProgressThreads(Context<Queue>& ctx) : ctx_(ctx) {}
    ~ProgressThreads() { stop(); }
    ProgressThreads(const ProgressThreads&) = delete;
    ProgressThreads& operator=(const ProgressThreads&) = delete;

    /// Starts `num_threads` threads (capped at the endpoint count).  `cpus`
    /// lists the cores to use, one per thread in order (wrapping); empty =
    /// no pinning.
    void start(size_t num_threads, std::vector<int> cpus = {}, Hook hook = {}) {
        stop();
        if (num_threads == 0) num_threads = 1;
        num_threads = std::min(num_threads, ctx_.num_endpoints());
        hook_ = std::move(hook);
        stop_.store(false);
        error_ = nullptr;
        for (size_t t = 0; t < num_threads; ++t) {
            std::vector<int> mine;
            if (!cpus.empty()) mine.push_back(cpus[t % cpus.size()]);
            threads_.emplace_back([this, t, num_threads, mine] { run(t, num_threads, mine); });
        }
    }

    /// Stops the threads after a final drain of every endpoint.
    void stop() {
        stop_.store(true);
        for (auto& th : threads_) th.join();
        threads_.clear();
    }

    bool running() const { return !threads_.empty(); }
    uint64_t callbacks_run() const { return callbacks_.load(std::memory_order_relaxed); }
    uint64_t sweeps() const { return sweeps_.load(std::memory_order_relaxed); }

    /// Rethrows the first exception a callback raised on a progress thread.
    void rethrow_if_failed() {
        std::lock_guard<std::mutex> g(mu_);
        if (error_) {
            auto e = error_;
            error_ = nullptr;
            std::rethrow_exception(e);
        }
    }

private:
    void run(size_t tid, size_t nthreads, std::vector<int> cpus) {
        if (!cpus.empty()) topology::bind_current_thread(cpus);
        std::vector<size_t> mine;
        for (size_t e = tid; e < ctx_.num_endpoints(); e += nthreads) mine.push_back(e);
        std::vector<queue::HostPollState> polls;
        for (size_t e : mine) polls.push_back(ctx_.poll_state(e));
        uint64_t local_sweeps = 0;
        try {
            while (!stop_.load(std::memory_order_relaxed)) {
                for (size_t i = 0; i < mine.size(); ++i) {
                    if (polls[i].ready()) {
                        callbacks_.fetch_add(ctx_.progress(mine[i]), std::memory_order_relaxed);
                        polls[i].refresh();
                    }
                    if (hook_) hook_(mine[i]);
                }
                if ((++local_sweeps & 1023u) == 0) sweeps_.fetch_add(1024, std::memory_order_relaxed);
            }
            for (size_t e : mine) callbacks_.fetch_add(ctx_.progress(e), std::memory_order_relaxed);
        } catch (...) {
            std::lock_guard<std::mutex> g(mu_);
            if (!error_) error_ = std::current_exception();
        }
    }

    Context<Queue>& ctx_;
    Hook hook_;
    std::vector<std::thread> threads_;
    std::atomic<bool> stop_{false};
    std::atomic<uint64_t> callbacks_{0};
    std::atomic<uint64_t> sweeps_{0};
    std::mutex mu_;
    std::exception_ptr error_;
};

}  // namespace kiwi::invoke
