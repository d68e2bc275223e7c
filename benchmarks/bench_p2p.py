"""Kernel-initiated P2P put / get / signal over NVLink vs NCCL send/recv
(the P2P latency and bandwidth sweep, 8 B - 64 MB, pairs of GPUs).

    torchrun --nproc-per-node N --master-addr 127.0.0.1 benchmarks/bench_p2p.py [--max-bytes 67108864]
    python benchmarks/bench_p2p.py --local     # one GPU: the put and all-to-all kernels on a one-rank heap

Ranks pair up (0<->1, 2<->3, ...).  For each size 8 B .. max (powers of two):
  * kiwi_pingpong: the initiator puts `size` bytes into its partner's heap and
    signals (release add on a flag word); the partner waits (acquire), puts back,
    signals.  One-way latency = round trip / 2 (device %globaltimer, p50).
  * kiwi_put_ll8 (payloads up to 4 KB): one warp, every 8-byte word carries
    4 data bytes and the sequence number -- no fence, no separate flag.
  * kiwi_put_bw: back-to-back puts of `size` bytes, one signal at the end.
  * kiwi_get: reads of `size` bytes from the partner's heap.
  Both rotate through a 256 MB region (larger than the 126 MB L2), one
  4 KB-aligned slot per repetition, so no repetition finds its lines cached
  (re-reading one address measured L1/L2 hits, ~0.1 us, not NVLink).
  * nccl_sendrecv: torch.distributed send/recv ping-pong of the same size,
    CUDA events, one-way = round trip / 2.
Data: seeded uniform uint8.  Every number is the max over ranks.

--local runs the data-plane kernels on one GPU with a one-rank heap (peer =
this GPU): a 64 MB put with release signal (put_bw, rotating over 256 MB of
this GPU's HBM) and 200 device all-to-all rounds; the mode a single-GPU
kernel profile of those two kernels uses.
"""
import argparse
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from kiwi_b200.parallel.p2p import SymmetricHeap  # noqa: E402
from kiwi_b200.utils import dist as kdist  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--max-bytes", type=int, default=64 << 20)
    ap.add_argument("--iters", type=int, default=200)
    ap.add_argument("--nccl", action="store_true", default=True)
    ap.add_argument("--local", action="store_true", help="one GPU, one-rank heap (peer = this GPU)")
    args = ap.parse_args()
    rank, world = kdist.init()
    if args.local:
        return local_kernels()
    assert world % 2 == 0, "run on an even number of ranks"
    peer = rank ^ 1
    initiator = rank % 2 == 0
    maxb = args.max_bytes
    region = max(maxb, 256 << 20)
    flag_off = 0
    src_off = 4096
    dst_off = src_off + region
    ll_base = dst_off + region + 4096
    heap = SymmetricHeap(ll_base + 65536)
    h = heap.native
    g = torch.Generator(device="cuda").manual_seed(1234 + rank)
    src = heap.tensor(src_off, [region], torch.uint8)
    src.copy_(torch.randint(0, 256, (region,), generator=g, device="cuda", dtype=torch.uint8))
    flag = heap.tensor(flag_off, [8], torch.int64)
    status = torch.zeros(2, dtype=torch.int32, device="cuda")
    sizes = [1 << i for i in range(3, int(np.log2(maxb)) + 1)]
    results = []
    for size in sizes:
        iters = args.iters if size <= (1 << 20) else max(10, args.iters // 10)
        lat = torch.zeros(iters, dtype=torch.int64, device="cuda")
        flag.zero_()
        torch.cuda.synchronize()
        kdist.barrier()
        h.pingpong(peer, initiator, size, iters, 5, src_off, dst_off, flag_off, lat, status, 132, 5_000_000_000)
        torch.cuda.synchronize()
        kdist.barrier()
        assert int(status[0].item()) == 0, f"pingpong timed out at {size}"
        one_way = float(np.percentile(lat.cpu().numpy(), 50)) / 2 / 1e3 if initiator else 0.0
        # LL8 (data + sequence per 8-byte word, no fence / flag) for payloads up to 4 KB
        ll8 = 0.0
        if size <= 4096:
            words = max(1, size // 4)
            ll_off = ll_base
            heap.tensor(ll_off, [words * 8], torch.uint8).zero_()
            lat2 = torch.zeros(iters, dtype=torch.int64, device="cuda")
            torch.cuda.synchronize()
            kdist.barrier()
            h.pingpong_ll8(peer, initiator, words, iters, 5, ll_off, lat2, status, 5_000_000_000)
            torch.cuda.synchronize()
            kdist.barrier()
            assert int(status[0].item()) == 0, f"ll8 pingpong timed out at {size}"
            ll8 = float(np.percentile(lat2.cpu().numpy(), 50)) / 2 / 1e3 if initiator else 0.0
        # bandwidth
        flag.zero_()
        el = torch.zeros(1, dtype=torch.int64, device="cuda")
        reps = max(1, min(1000, (256 << 20) // size))
        torch.cuda.synchronize()
        kdist.barrier()
        h.put_bw(peer, initiator, size, reps, src_off, dst_off, flag_off, 1, el, status, 132, 5_000_000_000, region)
        torch.cuda.synchronize()
        kdist.barrier()
        bw = size * reps / (el.item() / 1e9) / 1e9 if initiator and el.item() else 0.0
        # get
        glat = torch.zeros(20, dtype=torch.int64, device="cuda")
        h.get(peer, size, 20, src_off, dst_off, glat, 132, region)
        torch.cuda.synchronize()
        get_us = float(np.percentile(glat.cpu().numpy()[5:], 50)) / 1e3
        # NCCL send/recv ping-pong
        nccl_us = 0.0
        if args.nccl:
            buf = torch.empty(size, dtype=torch.uint8, device="cuda")
            n_it = 20 if size <= (1 << 20) else 5
            for it in range(n_it + 3):
                if it == 3:
                    torch.cuda.synchronize()
                    kdist.barrier()
                    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    s.record()
                if initiator:
                    dist.send(src[:size], peer)
                    dist.recv(buf, peer)
                else:
                    dist.recv(buf, peer)
                    dist.send(buf, peer)
            e.record()
            torch.cuda.synchronize()
            nccl_us = s.elapsed_time(e) / n_it / 2 * 1e3
        row = {"bytes": size,
               "kiwi_put_oneway_us": kdist.max_over_ranks(one_way),
               "kiwi_put_ll8_oneway_us": kdist.max_over_ranks(ll8),
               "kiwi_put_GBps": kdist.max_over_ranks(bw),
               "kiwi_get_us": kdist.max_over_ranks(get_us),
               "nccl_sendrecv_oneway_us": kdist.max_over_ranks(nccl_us)}
        results.append(row)
        if rank == 0:
            print("RESULT " + json.dumps({"bench": "p2p", "world": world, **row}), flush=True)
    # correctness: what the partner received equals what we sent
    kdist.barrier()
    mine = src[:maxb].clone()
    theirs = kdist.all_gather_objects(int(heap.tensor(dst_off, [maxb], torch.uint8).sum().item()))
    sums = kdist.all_gather_objects(int(mine.sum().item()))
    if rank == 0:
        ok = all(theirs[r ^ 1] == sums[r] for r in range(world))
        print("RESULT " + json.dumps({"bench": "p2p_check", "ok": ok}), flush=True)
    del heap
    dist.destroy_process_group()


def local_kernels():
    """put_bw and all2all_rounds on a one-rank heap; one RESULT line."""
    from kiwi_b200.parallel.collectives import DeviceCollectives

    size, region = 64 << 20, 256 << 20
    heap = SymmetricHeap(4096 + 2 * region + 4096)
    src_off, dst_off = 4096, 4096 + region
    g = torch.Generator(device="cuda").manual_seed(1234)
    heap.tensor(src_off, [region], torch.uint8).copy_(torch.randint(0, 256, (region,), generator=g,
                                                                    dtype=torch.uint8, device="cuda"))
    flag = heap.tensor(0, [8], torch.int64)
    status = torch.zeros(2, dtype=torch.int32, device="cuda")
    el = torch.zeros(1, dtype=torch.int64, device="cuda")
    gbps = []
    for _ in range(3):
        flag.zero_()
        heap.native.put_bw(0, True, size, 4, src_off, dst_off, 0, 1, el, status, 132, 5_000_000_000, region)
        torch.cuda.synchronize()
        gbps.append(size * 4 / (el.item() / 1e9) / 1e9)
    assert int(status[0].item()) == 0, status
    coll = DeviceCollectives()
    send = torch.tensor([5], dtype=torch.int32, device="cuda")
    lat = torch.zeros(200, dtype=torch.int64, device="cuda")
    out = coll.all2all(send, rounds=200, lat=lat)
    torch.cuda.synchronize()
    coll.check()
    assert out[-1, 0].item() == 5 + 199
    print("RESULT " + json.dumps({"bench": "p2p_local", "put_GBps_local": max(gbps),
                                  "all2all_round_us_world1": float(lat.float().median().item()) / 1e3}), flush=True)
    del heap


if __name__ == "__main__":
    main()
