// Host launchers for the kiwi::p2p kernels (csrc/p2p_gpu.cu).
#pragma once

#include <vector>

#include <cuda_runtime.h>

#include "kiwi/p2p/context.hpp"
#include "kiwi/p2p/counter.hpp"
#include "kiwi/p2p/heap.hpp"

namespace kiwi::p2p {

void launch_pingpong(const HeapView& h, int peer, bool initiator, uint64_t bytes, uint64_t iters, uint64_t warmup,
                     uint64_t src_off, uint64_t dst_off, uint64_t flag_off, uint64_t* lat_ns, uint32_t* status,
                     uint32_t max_blocks, uint64_t timeout_ns, cudaStream_t s);

void launch_pingpong_ll8(const HeapView& h, int peer, bool initiator, uint32_t words, uint64_t iters,
                         uint64_t warmup, uint64_t buf_off, uint64_t* lat_ns, uint32_t* status, uint64_t timeout_ns,
                         cudaStream_t s);

void launch_put_bw(const HeapView& h, int peer, bool sender, uint64_t bytes, uint64_t reps, uint64_t src_off,
                   uint64_t dst_off, uint64_t flag_off, uint64_t round, uint64_t* elapsed, uint32_t* status,
                   uint32_t max_blocks, uint64_t timeout_ns, cudaStream_t s, uint64_t region = 0);

void launch_get(const HeapView& h, int peer, uint64_t bytes, uint64_t reps, uint64_t src_off, uint64_t dst_off,
                uint64_t* lat_ns, uint32_t max_blocks, cudaStream_t s, uint64_t region = 0);

/// One block exercises the device API on caller-chosen ranges: put_block of
/// `bytes` from local offset 0 to (peer, off), get_block back from (peer, off)
/// into local offset `bytes`, and a signal on (peer, flag_off).  Exists for the
/// checked-mode tests; the caller keeps every range inside the mapped heap.
void launch_checked_ops(const HeapView& h, int peer, uint64_t off, uint64_t bytes, uint64_t flag_off, cudaStream_t s);

void launch_all_pairs(const HeapView& h, uint64_t data_off, uint64_t flag_off, uint64_t words, uint32_t round,
                      uint32_t* status, uint64_t timeout_ns, cudaStream_t s);

void launch_mc_broadcast(const HeapView& h, int root, uint64_t src_off, uint64_t dst_off, uint64_t bytes,
                         uint64_t flag_off, cudaStream_t s);

void launch_mc_allreduce_f32(const HeapView& h, uint64_t off, uint64_t count, cudaStream_t s);

void launch_wait_flag(const HeapView& h, uint64_t flag_off, uint64_t want, uint32_t* status, uint64_t timeout_ns,
                      cudaStream_t s);

void launch_heap_barrier(const HeapView& h, uint64_t flag_off, uint64_t round, uint32_t* status, uint64_t timeout_ns,
                         cudaStream_t s);

void launch_ce_put_selftest(const GContext& ctx, int dst, uint64_t src_off, uint64_t dst_off, uint64_t bytes,
                            uint32_t n, uint64_t flag_off, uint64_t counter_off, uint32_t* status,
                            uint64_t timeout_ns, cudaStream_t s);

// ---- device collectives (include/kiwi/p2p/collectives.cuh) ----

/// `rounds` all-to-all rounds of one u32 per rank pair (send == nullptr: barrier
/// rounds).  recv gets rounds x world values; lat_ns (optional) per-round time.
void launch_all2all_rounds(const HeapView& h, uint64_t ingress_off, const uint32_t* send, uint32_t* recv,
                           uint32_t* epoch_ctr, uint32_t* status, uint64_t timeout_ns, uint32_t rounds,
                           uint64_t* lat_ns, cudaStream_t s);

/// Waits (bounded) for a value nobody sends; records kTimeout in status.
void launch_coll_wait_only(const HeapView& h, uint64_t ingress_off, uint32_t epoch, int src, uint32_t* status,
                           uint64_t timeout_ns, uint64_t* waited_ns, cudaStream_t s);

/// Cooperative launch of the grid-barrier self test.
void launch_grid_barrier_test(unsigned long long* word, uint32_t* data, uint32_t blocks, uint32_t rounds,
                              uint32_t* status, uint64_t timeout_ns, uint64_t* elapsed_ns, cudaStream_t s);

/// Copy-engine ping-pong through the control plane (see csrc/p2p_gpu.cu).
void launch_ce_pingpong(const GContext& ctx, int peer, bool initiator, uint64_t bytes, uint32_t iters,
                        uint32_t warmup, uint64_t src_off, uint64_t dst_off, uint64_t flag_off, uint64_t* lat_ns,
                        uint32_t* status, uint64_t timeout_ns, cudaStream_t s);

/// Host-initiated copy-engine ping-pong (no kernel): a CPU thread issues
/// cudaMemcpyAsync into the peer's heap and the peer flag write, then a
/// stream wait on its own flag; returns per-round CPU round-trip ns
/// (initiator) and throws on a timeout.
std::vector<uint64_t> host_ce_pingpong(SymmetricHeap& heap, int peer, bool initiator, uint64_t bytes, uint32_t iters,
                                       uint32_t warmup, uint64_t src_off, uint64_t dst_off, uint64_t flag_off,
                                       double timeout_s);

/// Waits (one thread, bounded) for a completion counter to reach 1..steps.
void launch_counter_wait(const CounterView& c, uint32_t steps, uint64_t* seen_ns, uint32_t* status,
                         uint64_t timeout_ns, cudaStream_t s);

}  // namespace kiwi::p2p
