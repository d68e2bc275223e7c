// kiwi::p2p kernels: ping-pong put+signal latency, put bandwidth, get,
// NVLS broadcast / all-reduce, and the correctness kernels the tests use.
//
// Counterparts in the reference (AMDResearch/kiwi): apps/p2p/benchmarks/
// bench_latency.hip.cpp:50 (ping_pong_kernel), bench_bandwidth.hip.cpp:66,
// bench_loadstore_latency.hip.cpp:42-102 (plain peer stores + a system-scope
// flag, which on B200 is the product path rather than a baseline).
#include <cuda_runtime.h>

#include "kiwi/p2p/device.cuh"
#include "kiwi/p2p/p2p_ops.hpp"

namespace kiwi::p2p {

namespace {
KIWI_DEV void record_error(uint32_t* status, Status s, uint32_t info) {
    if (status) {
        atomicCAS(status, 0u, static_cast<uint32_t>(s));
        status[1] = info;
    }
}
}  // namespace

/// Ping-pong: the initiator puts `bytes` to the peer and signals; the responder
/// waits, puts the same number of bytes back and signals.  Every block copies
/// one slice and adds 1 to the peer's flag, so a side waits for
/// nblocks * (iteration + 1).
__global__ void __launch_bounds__(512) pingpong_kernel(HeapView h, int peer, int initiator, uint64_t bytes,
                                                       uint64_t iters, uint64_t warmup, uint64_t src_off,
                                                       uint64_t dst_off, uint64_t flag_off, uint64_t* lat_ns,
                                                       uint32_t* status, uint64_t timeout_ns) {
    __shared__ int s_abort;
    const uint32_t nb = gridDim.x;
    const uint64_t slice = round_up((bytes + nb - 1) / nb, 16);
    const uint64_t my_off = slice * blockIdx.x;
    const uint64_t my_bytes = my_off >= bytes ? 0 : (bytes - my_off < slice ? bytes - my_off : slice);
    const uint64_t* my_flag = reinterpret_cast<const uint64_t*>(h.base[h.rank] + flag_off);
    if (threadIdx.x == 0) s_abort = 0;
    __syncthreads();
    for (uint64_t i = 0; i < iters + warmup; ++i) {
        const uint64_t want = static_cast<uint64_t>(nb) * (i + 1);
        uint64_t t0 = 0;
        if (!initiator) {
            if (threadIdx.x == 0 && wait(my_flag, Cmp::kGe, want, timeout_ns) != Status::kOk) {
                record_error(status, Status::kTimeout, static_cast<uint32_t>(i));
                s_abort = 1;
            }
            __syncthreads();
            if (s_abort) return;
        } else if (blockIdx.x == 0 && threadIdx.x == 0) {
            t0 = ptx::globaltimer();
        }
        coop_copy(h.base[peer] + dst_off + my_off, h.base[h.rank] + src_off + my_off, my_bytes, threadIdx.x,
                  blockDim.x);
        __syncthreads();
        if (threadIdx.x == 0) signal(h, peer, flag_off, 1, SignalOp::kAdd);
        if (initiator) {
            if (threadIdx.x == 0) {
                if (wait(my_flag, Cmp::kGe, want, timeout_ns) != Status::kOk) {
                    record_error(status, Status::kTimeout, static_cast<uint32_t>(i));
                    s_abort = 1;
                } else if (blockIdx.x == 0 && i >= warmup) {
                    lat_ns[i - warmup] = ptx::globaltimer() - t0;
                }
            }
            __syncthreads();
            if (s_abort) return;
        }
    }
}

/// LL8 ping-pong (one warp, messages of `words` 32-bit words): data and
/// sequence travel together, so there is no fence and no separate flag.
__global__ void pingpong_ll8_kernel(HeapView h, int peer, int initiator, uint32_t words, uint64_t iters,
                                    uint64_t warmup, uint64_t buf_off, uint64_t* lat_ns, uint32_t* status,
                                    uint64_t timeout_ns) {
    __shared__ uint32_t msg[1024];
    const uint64_t* inbox = reinterpret_cast<const uint64_t*>(h.base[h.rank] + buf_off);
    for (uint32_t i = threadIdx.x; i < words; i += 32) msg[i] = i * 2654435761u;
    __syncwarp();
    for (uint64_t it = 0; it < iters + warmup; ++it) {
        const uint32_t seq = static_cast<uint32_t>(it + 1);
        uint64_t t0 = 0;
        if (initiator) {
            if (threadIdx.x == 0) t0 = ptx::globaltimer();
            put_ll8_warp(h, peer, buf_off, msg, words, seq);
            if (recv_ll8_warp(inbox, msg, words, seq, timeout_ns) != Status::kOk) {
                if (threadIdx.x == 0) record_error(status, Status::kTimeout, static_cast<uint32_t>(it));
                return;
            }
            if (threadIdx.x == 0 && it >= warmup) lat_ns[it - warmup] = ptx::globaltimer() - t0;
        } else {
            if (recv_ll8_warp(inbox, msg, words, seq, timeout_ns) != Status::kOk) {
                if (threadIdx.x == 0) record_error(status, Status::kTimeout, static_cast<uint32_t>(it));
                return;
            }
            put_ll8_warp(h, peer, buf_off, msg, words, seq);
        }
        __syncwarp();
    }
}

void launch_pingpong_ll8(const HeapView& h, int peer, bool initiator, uint32_t words, uint64_t iters,
                         uint64_t warmup, uint64_t buf_off, uint64_t* lat_ns, uint32_t* status, uint64_t timeout_ns,
                         cudaStream_t s) {
    if (words == 0 || words > 1024) throw kiwi::error("pingpong_ll8: 1..1024 words");
    pingpong_ll8_kernel<<<1, 32, 0, s>>>(h, peer, initiator ? 1 : 0, words, iters, warmup, buf_off, lat_ns, status,
                                         timeout_ns);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

/// One-directional put bandwidth: `reps` back-to-back puts of `bytes`, one
/// signal per block at the end; the receiver answers with one signal.
/// Offset of repetition r when `region` bytes are rotated through in slots of
/// round_up(bytes, 4096) (region 0: no rotation).  Benchmarks rotate through
/// more than the 126 MB L2 so that no repetition finds its lines cached.
KIWI_DEV uint64_t rep_offset(uint64_t r, uint64_t bytes, uint64_t region) {
    const uint64_t stride = round_up(bytes, 4096);
    const uint64_t slots = region >= stride ? region / stride : 1;
    return (r % slots) * stride;
}

__global__ void __launch_bounds__(512) put_bw_kernel(HeapView h, int peer, int sender, uint64_t bytes, uint64_t reps,
                                                     uint64_t src_off, uint64_t dst_off, uint64_t flag_off,
                                                     uint64_t round, uint64_t* elapsed_ns, uint32_t* status,
                                                     uint64_t timeout_ns, uint64_t region) {
    const uint32_t nb = gridDim.x;
    const uint64_t* my_flag = reinterpret_cast<const uint64_t*>(h.base[h.rank] + flag_off);
    if (!sender) {
        if (blockIdx.x == 0 && threadIdx.x == 0) {
            if (wait(my_flag, Cmp::kGe, static_cast<uint64_t>(nb) * round, timeout_ns) != Status::kOk) {
                record_error(status, Status::kTimeout, 0);
                return;
            }
            signal(h, peer, flag_off, 1, SignalOp::kAdd);
        }
        return;
    }
    const uint64_t slice = round_up((bytes + nb - 1) / nb, 16);
    const uint64_t my_off = slice * blockIdx.x;
    const uint64_t my_bytes = my_off >= bytes ? 0 : (bytes - my_off < slice ? bytes - my_off : slice);
    const uint64_t t0 = ptx::globaltimer();
    for (uint64_t r = 0; r < reps; ++r) {
        const uint64_t ro = rep_offset(r, bytes, region);
        coop_copy(h.base[peer] + dst_off + ro + my_off, h.base[h.rank] + src_off + ro + my_off, my_bytes,
                  threadIdx.x, blockDim.x);
    }
    __syncthreads();
    if (threadIdx.x == 0) signal(h, peer, flag_off, 1, SignalOp::kAdd);
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        if (wait(my_flag, Cmp::kGe, round, timeout_ns) != Status::kOk) {
            record_error(status, Status::kTimeout, 1);
            return;
        }
        *elapsed_ns = ptx::globaltimer() - t0;
    }
}

/// Get: `reps` reads of `bytes` from the peer's heap into local memory.
__global__ void __launch_bounds__(512) get_kernel(HeapView h, int peer, uint64_t bytes, uint64_t reps,
                                                  uint64_t src_off, uint64_t dst_off, uint64_t* lat_ns,
                                                  uint64_t region) {
    const uint32_t nb = gridDim.x;
    const uint64_t slice = round_up((bytes + nb - 1) / nb, 16);
    const uint64_t my_off = slice * blockIdx.x;
    const uint64_t my_bytes = my_off >= bytes ? 0 : (bytes - my_off < slice ? bytes - my_off : slice);
    for (uint64_t r = 0; r < reps; ++r) {
        const uint64_t ro = rep_offset(r, bytes, region);
        const uint64_t t0 = ptx::globaltimer();
        coop_copy(h.base[h.rank] + dst_off + ro + my_off, h.base[peer] + src_off + ro + my_off, my_bytes,
                  threadIdx.x, blockDim.x);
        __syncthreads();
        if (blockIdx.x == 0 && threadIdx.x == 0) lat_ns[r] = ptx::globaltimer() - t0;
    }
}

__global__ void checked_ops_kernel(HeapView h, int peer, uint64_t off, uint64_t bytes, uint64_t flag_off) {
    put_block(h, peer, off, h.base[h.rank], bytes);
    __syncthreads();
    get_block(h, peer, off, h.base[h.rank] + bytes, bytes);
    __syncthreads();
    if (threadIdx.x == 0) signal(h, peer, flag_off, 1, SignalOp::kAdd);
}

/// Every rank stores (rank+1) * (i+1) into its slot of every peer, signals them,
/// then waits for all peers and checks what arrived (all-pairs put test).
__global__ void all_pairs_kernel(HeapView h, uint64_t data_off, uint64_t flag_off, uint64_t words, uint32_t round,
                                 uint32_t* status, uint64_t timeout_ns) {
    const int me = h.rank;
    for (int k = 1; k < h.world; ++k) {
        const int peer = (me + k) % h.world;
        uint64_t* dst = reinterpret_cast<uint64_t*>(h.base[peer] + data_off) + static_cast<uint64_t>(me) * words;
        for (uint64_t w = threadIdx.x; w < words; w += blockDim.x) dst[w] = (static_cast<uint64_t>(me + 1) << 32) | (w + round);
        __syncthreads();
        if (threadIdx.x == 0) signal(h, peer, flag_off + 8 * me, round, SignalOp::kSet);
    }
    __syncthreads();
    for (int p = 0; p < h.world; ++p) {
        if (p == me) continue;
        if (threadIdx.x == 0) {
            const uint64_t* f = reinterpret_cast<const uint64_t*>(h.base[me] + flag_off + 8 * p);
            if (wait(f, Cmp::kGe, round, timeout_ns) != Status::kOk) record_error(status, Status::kTimeout, p);
        }
        __syncthreads();
        const uint64_t* src = reinterpret_cast<const uint64_t*>(h.base[me] + data_off) + static_cast<uint64_t>(p) * words;
        for (uint64_t w = threadIdx.x; w < words; w += blockDim.x) {
            if (src[w] != ((static_cast<uint64_t>(p + 1) << 32) | (w + round))) record_error(status, Status::kCorrupt, p);
        }
    }
}

/// NVLS: rank `root` broadcasts `bytes` from its heap at src_off into every
/// rank's heap at dst_off with multimem.st, then bumps every rank's flag.
__global__ void __launch_bounds__(512) mc_broadcast_kernel(HeapView h, int root, uint64_t src_off, uint64_t dst_off,
                                                           uint64_t bytes, uint64_t flag_off) {
    if (h.rank != root) return;
    const uint64_t n = bytes / 16;
    const uint4* s = reinterpret_cast<const uint4*>(h.base[h.rank] + src_off);
    uint4* d = reinterpret_cast<uint4*>(h.mc + dst_off);
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        mc_store_v4(d + i, ptx::ld_v4(s + i));
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        ptx::fence_acq_rel_sys();
        mc_red_add_u64(h.mc + flag_off, 1);
    }
}

/// NVLS all-reduce of fp32: every rank reads the multicast sum of its slice and
/// stores it back with multimem.st (one-shot, each rank owns 1/world of the data).
__global__ void __launch_bounds__(512) mc_allreduce_f32_kernel(HeapView h, uint64_t off, uint64_t count) {
    const uint64_t nvec = count / 4;
    const uint64_t per = (nvec + h.world - 1) / h.world;
    const uint64_t begin = per * h.rank;
    const uint64_t end = begin + per < nvec ? begin + per : nvec;
    float4* base = reinterpret_cast<float4*>(h.mc + off);
    for (uint64_t i = begin + blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < end;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const float4 s = mc_reduce_add_f32_v4(base + i);
        mc_store_v4(base + i, make_uint4(__float_as_uint(s.x), __float_as_uint(s.y), __float_as_uint(s.z),
                                         __float_as_uint(s.w)));
    }
}

/// Waits on this rank's flag (used after an NVLS broadcast / all-reduce phase).
__global__ void wait_flag_kernel(HeapView h, uint64_t flag_off, uint64_t want, uint32_t* status, uint64_t timeout_ns) {
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        const uint64_t* f = reinterpret_cast<const uint64_t*>(h.base[h.rank] + flag_off);
        if (wait(f, Cmp::kGe, want, timeout_ns) != Status::kOk) record_error(status, Status::kTimeout, 0);
    }
}

/// Cross-rank barrier on the heap: add 1 to flag_off + 8*me on every peer, wait for all.
__global__ void heap_barrier_kernel(HeapView h, uint64_t flag_off, uint64_t round, uint32_t* status,
                                    uint64_t timeout_ns) {
    const int t = threadIdx.x;
    if (t < h.world && t != h.rank) ptx::st_release_sys_u64(h.base[t] + flag_off + 8 * h.rank, round);
    __syncwarp();
    if (t < h.world && t != h.rank) {
        const uint64_t* f = reinterpret_cast<const uint64_t*>(h.base[h.rank] + flag_off + 8 * t);
        if (wait(f, Cmp::kGe, round, timeout_ns) != Status::kOk) record_error(status, Status::kTimeout, t);
    }
}

// ---------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------

static uint32_t blocks_for(uint64_t bytes, uint32_t max_blocks) {
    const uint64_t b = (bytes + 65535) / 65536;  // 64 KB per block
    return static_cast<uint32_t>(b < 1 ? 1 : (b > max_blocks ? max_blocks : b));
}

void launch_pingpong(const HeapView& h, int peer, bool initiator, uint64_t bytes, uint64_t iters, uint64_t warmup,
                     uint64_t src_off, uint64_t dst_off, uint64_t flag_off, uint64_t* lat_ns, uint32_t* status,
                     uint32_t max_blocks, uint64_t timeout_ns, cudaStream_t s) {
    const uint32_t nb = blocks_for(bytes, max_blocks);
    const uint32_t threads = bytes <= 4096 ? 128 : 512;
    pingpong_kernel<<<nb, threads, 0, s>>>(h, peer, initiator ? 1 : 0, bytes, iters, warmup, src_off, dst_off,
                                           flag_off, lat_ns, status, timeout_ns);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

void launch_put_bw(const HeapView& h, int peer, bool sender, uint64_t bytes, uint64_t reps, uint64_t src_off,
                   uint64_t dst_off, uint64_t flag_off, uint64_t round, uint64_t* elapsed, uint32_t* status,
                   uint32_t max_blocks, uint64_t timeout_ns, cudaStream_t s, uint64_t region) {
    const uint32_t nb = sender ? blocks_for(bytes, max_blocks) : 1;
    put_bw_kernel<<<nb, 512, 0, s>>>(h, peer, sender ? 1 : 0, bytes, reps, src_off, dst_off, flag_off, round,
                                     elapsed, status, timeout_ns, region);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

void launch_get(const HeapView& h, int peer, uint64_t bytes, uint64_t reps, uint64_t src_off, uint64_t dst_off,
                uint64_t* lat_ns, uint32_t max_blocks, cudaStream_t s, uint64_t region) {
    const uint32_t nb = blocks_for(bytes, max_blocks);
    get_kernel<<<nb, bytes <= 4096 ? 128 : 512, 0, s>>>(h, peer, bytes, reps, src_off, dst_off, lat_ns, region);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

void launch_checked_ops(const HeapView& h, int peer, uint64_t off, uint64_t bytes, uint64_t flag_off, cudaStream_t s) {
    checked_ops_kernel<<<1, 256, 0, s>>>(h, peer, off, bytes, flag_off);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

void launch_all_pairs(const HeapView& h, uint64_t data_off, uint64_t flag_off, uint64_t words, uint32_t round,
                      uint32_t* status, uint64_t timeout_ns, cudaStream_t s) {
    all_pairs_kernel<<<1, 256, 0, s>>>(h, data_off, flag_off, words, round, status, timeout_ns);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

void launch_mc_broadcast(const HeapView& h, int root, uint64_t src_off, uint64_t dst_off, uint64_t bytes,
                         uint64_t flag_off, cudaStream_t s) {
    if (!h.mc) throw kiwi::error("kiwi::p2p: heap has no multicast mapping");
    if (bytes % 16) throw kiwi::error("kiwi::p2p: multicast broadcast needs a multiple of 16 bytes");
    mc_broadcast_kernel<<<blocks_for(bytes, 132), 512, 0, s>>>(h, root, src_off, dst_off, bytes, flag_off);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

void launch_mc_allreduce_f32(const HeapView& h, uint64_t off, uint64_t count, cudaStream_t s) {
    if (!h.mc) throw kiwi::error("kiwi::p2p: heap has no multicast mapping");
    if (count % 4) throw kiwi::error("kiwi::p2p: all-reduce count must be a multiple of 4");
    mc_allreduce_f32_kernel<<<blocks_for(count * 4 / h.world, 132), 512, 0, s>>>(h, off, count);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

void launch_wait_flag(const HeapView& h, uint64_t flag_off, uint64_t want, uint32_t* status, uint64_t timeout_ns,
                      cudaStream_t s) {
    wait_flag_kernel<<<1, 32, 0, s>>>(h, flag_off, want, status, timeout_ns);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

void launch_heap_barrier(const HeapView& h, uint64_t flag_off, uint64_t round, uint32_t* status, uint64_t timeout_ns,
                         cudaStream_t s) {
    heap_barrier_kernel<<<1, 32, 0, s>>>(h, flag_off, round, status, timeout_ns);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

}  // namespace kiwi::p2p

// ---------------------------------------------------------------------------
// Control-plane self test: one warp posts `n` copy-engine puts of `bytes`
// (src_off -> dst_off + i*bytes on rank `dst`), each followed by a flag the
// proxy writes; the warp waits (bounded) for every flag and the local counter.
// ---------------------------------------------------------------------------
#include "kiwi/p2p/counter.hpp"
#include "kiwi/p2p/ghandle.cuh"

namespace kiwi::p2p {

__global__ void ce_put_selftest_kernel(GContext ctx, int dst, uint64_t src_off, uint64_t dst_off, uint64_t bytes,
                                       uint32_t n, uint64_t flag_off, uint64_t counter_off, uint32_t* status,
                                       uint64_t timeout_ns) {
    GHandle g(ctx, 0);
    for (uint32_t i = 0; i < n; ++i) {
        CePutDesc d{};
        d.dst_rank = static_cast<uint32_t>(dst);
        d.flag_rank = static_cast<uint32_t>(dst);
        d.dst_off = dst_off + i * bytes;
        d.src_off = src_off;
        d.bytes = bytes;
        d.flag_off = flag_off;
        d.flag_value = i + 1;
        d.counter_off = counter_off;
        d.counter_value = i + 1;
        if (g.post_ce_put(d, timeout_ns) != Status::kOk) {
            if (ptx::lane_id() == 0) status[0] = 1;
            return;
        }
    }
    if (dst == ctx.heap.rank) {
        if (g.wait_local(flag_off, Cmp::kGe, n, timeout_ns) != Status::kOk) {
            if (ptx::lane_id() == 0) status[0] = 2;
            return;
        }
    }
    if (g.wait_local(counter_off, Cmp::kGe, n, timeout_ns) != Status::kOk) {
        if (ptx::lane_id() == 0) status[0] = 3;
        return;
    }
    if (g.post_host_signal(ctx.heap.rank, flag_off + 8, 0xabcdull, timeout_ns) != Status::kOk) {
        if (ptx::lane_id() == 0) status[0] = 4;
        return;
    }
    if (g.wait_local(flag_off + 8, Cmp::kEq, 0xabcdull, timeout_ns) != Status::kOk) {
        if (ptx::lane_id() == 0) status[0] = 5;
    }
}

/// Copy-engine ping-pong (the B200 counterpart of the reference's invoke ->
/// host SDMA ping-pong, examples/invoke/invoke_sdma_ping_pong.hip.cpp:501-553):
/// in round i the initiator's warp posts a copy-engine put of `bytes` to the
/// peer with flag value i (a proxy thread issues cudaMemcpyAsync and the flag
/// write on its copy stream), then waits for the peer's put back; the
/// responder waits for round i and answers the same way.  lat_ns[i - warmup]
/// = the initiator's round trip (device %globaltimer).
__global__ void ce_pingpong_kernel(GContext ctx, int peer, int initiator, uint64_t bytes, uint32_t iters,
                                   uint32_t warmup, uint64_t src_off, uint64_t dst_off, uint64_t flag_off,
                                   uint64_t* lat_ns, uint32_t* status, uint64_t timeout_ns) {
    GHandle g(ctx, 0);
    auto put_back = [&](uint32_t i) {
        CePutDesc d{};
        d.dst_rank = static_cast<uint32_t>(peer);
        d.flag_rank = static_cast<uint32_t>(peer);
        d.dst_off = dst_off;
        d.src_off = src_off;
        d.bytes = bytes;
        d.flag_off = flag_off;
        d.flag_value = i;
        d.counter_off = flag_off + 8;  // local completion counter (unused by the ping-pong)
        d.counter_value = 0;
        return g.post_ce_put(d, timeout_ns);
    };
    for (uint32_t i = 1; i <= iters + warmup; ++i) {
        const uint64_t t0 = ptx::globaltimer();
        if (initiator) {
            if (put_back(i) != Status::kOk) {
                if (ptx::lane_id() == 0) status[0] = 1;
                return;
            }
        }
        if (g.wait_local(flag_off, Cmp::kGe, i, timeout_ns) != Status::kOk) {
            if (ptx::lane_id() == 0) {
                status[0] = 2;
                status[1] = i;
            }
            return;
        }
        if (!initiator) {
            if (put_back(i) != Status::kOk) {
                if (ptx::lane_id() == 0) status[0] = 3;
                return;
            }
        } else if (i > warmup && ptx::lane_id() == 0) {
            lat_ns[i - 1 - warmup] = ptx::globaltimer() - t0;
        }
    }
}

void launch_ce_pingpong(const GContext& ctx, int peer, bool initiator, uint64_t bytes, uint32_t iters,
                        uint32_t warmup, uint64_t src_off, uint64_t dst_off, uint64_t flag_off, uint64_t* lat_ns,
                        uint32_t* status, uint64_t timeout_ns, cudaStream_t s) {
    ce_pingpong_kernel<<<1, 32, 0, s>>>(ctx, peer, initiator ? 1 : 0, bytes, iters, warmup, src_off, dst_off,
                                        flag_off, lat_ns, status, timeout_ns);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

/// Completion-counter test kernel: one thread waits (bounded) for the counter
/// to reach 1, 2, ..., steps, recording when each value was seen.
__global__ void counter_wait_kernel(CounterView c, uint32_t steps, uint64_t* seen_ns, uint32_t* status,
                                    uint64_t timeout_ns) {
    for (uint32_t i = 1; i <= steps; ++i) {
        if (c.poll(i, timeout_ns) != Status::kOk) {
            status[0] = static_cast<uint32_t>(Status::kTimeout);
            status[1] = i;
            return;
        }
        seen_ns[i - 1] = ptx::globaltimer();
    }
}

void launch_counter_wait(const CounterView& c, uint32_t steps, uint64_t* seen_ns, uint32_t* status,
                         uint64_t timeout_ns, cudaStream_t s) {
    counter_wait_kernel<<<1, 1, 0, s>>>(c, steps, seen_ns, status, timeout_ns);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

void launch_ce_put_selftest(const GContext& ctx, int dst, uint64_t src_off, uint64_t dst_off, uint64_t bytes,
                            uint32_t n, uint64_t flag_off, uint64_t counter_off, uint32_t* status,
                            uint64_t timeout_ns, cudaStream_t s) {
    ce_put_selftest_kernel<<<1, 32, 0, s>>>(ctx, dst, src_off, dst_off, bytes, n, flag_off, counter_off, status,
                                            timeout_ns);
    KIWI_CUDA_CHECK(cudaGetLastError());
}

}  // namespace kiwi::p2p
