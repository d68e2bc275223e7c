// Host side of a benchmark kernel on a thread of its own.
//
// launch_with_server() starts the thread that serves a kernel (pops its
// messages, writes its acknowledgements) BEFORE the kernel is launched, so a
// tool that blocks inside the launch call (a profiler replaying the kernel)
// cannot leave the kernel without its host side until the kernel's bounded
// waits run out.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <exception>
#include <thread>

#include "kiwi/common.hpp"
#include "kiwi/topology.hpp"

namespace kiwi::bench {

/// Runs `serve(launched, quit)` on a new thread (on the caller's device,
/// pinned to `cpu` when it is >= 0) and then `launch()` on the calling
/// thread.  `serve` polls until its work is done; it may ask whether the
/// launch has returned (`launched`, so an empty stream before the launch is
/// not taken for a finished kernel) and must return when `quit` turns true
/// (the launch threw).  Exceptions of either side are rethrown here.
template <typename Launch, typename Serve>
void launch_with_server(int cpu, Launch&& launch, Serve&& serve) {
    std::atomic<bool> launched{false}, quit{false};
    std::exception_ptr err;
    int dev = 0;
    KIWI_CUDA_CHECK(cudaGetDevice(&dev));
    std::thread th([&] {
        try {
            KIWI_CUDA_CHECK(cudaSetDevice(dev));
            if (cpu >= 0) topology::bind_current_thread({cpu});
            serve(launched, quit);
        } catch (...) {
            err = std::current_exception();
        }
    });
    try {
        launch();
    } catch (...) {
        quit.store(true);
        th.join();
        throw;
    }
    launched.store(true, std::memory_order_release);
    th.join();
    if (err) std::rethrow_exception(err);
}

/// True when `stream` has no work left; only asked after the launch returned.
inline bool stream_idle(cudaStream_t stream, const std::atomic<bool>& launched) {
    return launched.load(std::memory_order_acquire) && cudaStreamQuery(stream) != cudaErrorNotReady;
}

}  // namespace kiwi::bench
