// Kernels and launchers of the kiwi::p2p device collectives
// (include/kiwi/p2p/collectives.cuh): count all-to-all and barrier rounds over
// the symmetric heap, a grid-barrier self test and a wait that is meant to run
// out (timeout test).  Reference parity: apps/ep/all2all.hip.{hpp,cpp},
// apps/ep/barrier.hpp, apps/ep/benchmarks/bench_ep_collectives.hip.cpp:234-250
// of AMDResearch/kiwi.
#include <cuda_runtime.h>

#include "kiwi/p2p/collectives.cuh"
#include "kiwi/p2p/p2p_ops.hpp"

namespace kiwi::p2p {
namespace {

KIWI_DEV void coll_record(uint32_t* status, Status s, uint32_t info) {
    if (status && atomicCAS(status, 0u, static_cast<uint32_t>(s)) == 0u) status[1] = info;
}

/// `rounds` back-to-back all-to-all rounds.  Round r sends send[d] + r to rank
/// d and stores what rank s sent in recv[r * world + s]; lat_ns[r] (optional)
/// gets the round's device time.  epoch_ctr holds the last finished epoch.
__global__ void all2all_rounds_kernel(HeapView h, uint64_t ingress_off, const uint32_t* send, uint32_t* recv,
                                      uint32_t* epoch_ctr, uint32_t* status, uint64_t timeout_ns, uint32_t rounds,
                                      uint64_t* lat_ns, int with_values) {
    __shared__ uint32_t s_send[kMaxRanks];
    const uint32_t base = *reinterpret_cast<volatile uint32_t*>(epoch_ctr);
    for (uint32_t r = 0; r < rounds; ++r) {
        const uint32_t epoch = base + 1 + r;
        if (with_values && threadIdx.x < static_cast<uint32_t>(h.world)) s_send[threadIdx.x] = send[threadIdx.x] + r;
        const uint64_t t0 = ptx::globaltimer();
        int bad = -1;
        const Status st = all2all_block(h, ingress_off, epoch, with_values ? s_send : nullptr,
                                        with_values ? recv + static_cast<uint64_t>(r) * h.world : nullptr,
                                        timeout_ns, &bad);
        if (threadIdx.x == 0 && lat_ns) lat_ns[r] = ptx::globaltimer() - t0;
        if (st != Status::kOk) {
            if (threadIdx.x == 0) {
                coll_record(status, st, static_cast<uint32_t>(bad));
                *epoch_ctr = epoch;  // keep the count in step with the peers that did post
            }
            return;
        }
    }
    if (threadIdx.x == 0) *epoch_ctr = base + rounds;
}

/// Waits for a value of round `epoch` from rank `src` that nobody sends.
__global__ void coll_wait_only_kernel(HeapView h, uint64_t ingress_off, uint32_t epoch, int src, uint32_t* status,
                                      uint64_t timeout_ns, uint64_t* waited_ns) {
    uint32_t v = 0;
    const uint64_t t0 = ptx::globaltimer();
    const Status st = all2all_wait(h, ingress_off, epoch, src, v, timeout_ns);
    *waited_ns = ptx::globaltimer() - t0;
    if (st != Status::kOk) coll_record(status, st, static_cast<uint32_t>(src));
}

/// Grid-barrier self test: in round r every block writes r into its slot,
/// syncs, checks its neighbour's slot, syncs again.
__global__ void grid_barrier_test_kernel(unsigned long long* word, uint32_t* data, uint32_t rounds, uint32_t* status,
                                         uint64_t timeout_ns, uint64_t* elapsed_ns) {
    GridBarrier gb{word};
    const uint32_t nb = gridDim.x;
    const uint64_t t0 = ptx::globaltimer();
    for (uint32_t r = 1; r <= rounds; ++r) {
        if (threadIdx.x == 0) reinterpret_cast<volatile uint32_t*>(data)[blockIdx.x] = r;
        if (gb.sync(timeout_ns) != Status::kOk) {
            if (threadIdx.x == 0) coll_record(status, Status::kTimeout, r);
            return;
        }
        if (threadIdx.x == 0) {
            const uint32_t got = reinterpret_cast<volatile uint32_t*>(data)[(blockIdx.x + 1) % nb];
            if (got != r) coll_record(status, Status::kCorrupt, r);
        }
        if (gb.sync(timeout_ns) != Status::kOk) {
            if (threadIdx.x == 0) coll_record(status, Status::kTimeout, r);
            return;
        }
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) *elapsed_ns = ptx::globaltimer() - t0;
}

}  // namespace

void launch_all2all_rounds(const HeapView& h, uint64_t ingress_off, const uint32_t* send, uint32_t* recv,
                           uint32_t* epoch_ctr, uint32_t* status, uint64_t timeout_ns, uint32_t rounds,
                           uint64_t* lat_ns, cudaStream_t s) {
    if (ingress_off % 64) throw kiwi::error("kiwi::p2p collectives: ingress offset must be 64-byte aligned");
    all2all_rounds_kernel<<<1, 32, 0, s>>>(h, ingress_off, send, recv, epoch_ctr, status, timeout_ns, rounds, lat_ns,
                                          send != nullptr ? 1 : 0);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

void launch_coll_wait_only(const HeapView& h, uint64_t ingress_off, uint32_t epoch, int src, uint32_t* status,
                           uint64_t timeout_ns, uint64_t* waited_ns, cudaStream_t s) {
    coll_wait_only_kernel<<<1, 1, 0, s>>>(h, ingress_off, epoch, src, status, timeout_ns, waited_ns);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

void launch_grid_barrier_test(unsigned long long* word, uint32_t* data, uint32_t blocks, uint32_t rounds,
                              uint32_t* status, uint64_t timeout_ns, uint64_t* elapsed_ns, cudaStream_t s) {
    int dev = 0, coop = 0, per_sm = 0, sms = 0;
    KIWI_CUDA_CHECK(cudaGetDevice(&dev));
    KIWI_CUDA_CHECK(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev));
    KIWI_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    KIWI_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, grid_barrier_test_kernel, 128, 0));
    if (!coop) throw kiwi::error("grid_barrier_test: device has no cooperative launch");
    if (blocks == 0 || blocks > static_cast<uint32_t>(per_sm * sms)) {
        throw kiwi::error("grid_barrier_test: blocks must be 1.." + std::to_string(per_sm * sms) +
                          " (co-resident limit)");
    }
    void* args[] = {&word, &data, &rounds, &status, &timeout_ns, &elapsed_ns};
    KIWI_CUDA_CHECK(cudaLaunchCooperativeKernel(reinterpret_cast<void*>(grid_barrier_test_kernel), dim3(blocks),
                                                dim3(128), args, 0, s));
}

}  // namespace kiwi::p2p
