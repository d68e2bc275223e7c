"""Two-GPU ping-pong three ways (the B200 counterpart of the reference's
invoke SDMA ping-pong example, examples/invoke/invoke_sdma_ping_pong.hip.cpp):

* device: the kernel stores the payload into the peer's heap over NVLink and
  signals it (release add); the peer waits (acquire) and answers.
* invoke: the kernel posts a copy-engine put descriptor on its invoke control
  queue; a host proxy thread issues cudaMemcpyAsync into the peer's heap and
  the peer's flag write (cuStreamWriteValue64) on its copy stream; the peer's
  kernel waits for the flag and answers the same way.
* host: no kernel; each rank's CPU thread issues the copy and the flag write
  and makes its stream wait for its own flag (cuStreamWaitValue64).

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 examples/python/ce_pingpong.py [--max-bytes N]

Rank 0 prints one RESULT line per size: one-way latency (round trip / 2, p50)
of each mode; device and invoke are timed on the GPU (%globaltimer), host on
the CPU.  After every size and mode both ranks check that their destination
holds the peer's source bytes.
"""
import argparse
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
import numpy as np  # noqa: E402
import torch  # noqa: E402

import kiwi_b200  # noqa: E402
from kiwi_b200.parallel.p2p import SymmetricHeap  # noqa: E402
from kiwi_b200.utils import dist as kdist  # noqa: E402

FLAG_OFF = 0
SRC_OFF = 1 << 20


def run(sizes, iters=50, warmup=5, timeout_s=10.0):
    """Runs every mode for every size on a two-rank job; returns rank 0's rows."""
    C = kiwi_b200.native()
    rank, world = kdist.rank(), kdist.world_size()
    assert world == 2, "run on exactly two ranks"
    peer, initiator = 1 - rank, rank == 0
    maxb = max(sizes)
    dst_off = SRC_OFF + ((maxb + 4095) // 4096) * 4096
    heap = SymmetricHeap(dst_off + maxb + 4096)
    g = torch.Generator(device="cuda").manual_seed(77 + rank)
    src = heap.tensor(SRC_OFF, [maxb], torch.uint8)
    src.copy_(torch.randint(0, 256, (maxb,), generator=g, device="cuda", dtype=torch.uint8))
    flags = heap.tensor(FLAG_OFF, [16], torch.int64)
    ctx = C.p2p.Context(heap.native, 1)
    ctx.spawn_proxy_threads(1)
    status = torch.zeros(2, dtype=torch.int32, device="cuda")
    rows = []
    try:
        for size in sizes:
            row = {"bytes": size}
            for mode in ("device", "invoke", "host"):
                flags.zero_()
                heap.tensor(dst_off, [maxb], torch.uint8).zero_()
                status.zero_()
                torch.cuda.synchronize()
                kdist.barrier()
                lat = torch.zeros(iters, dtype=torch.int64, device="cuda")
                if mode == "device":
                    heap.native.pingpong(peer, initiator, size, iters, warmup, SRC_OFF, dst_off, FLAG_OFF, lat,
                                         status, 132, int(timeout_s * 1e9))
                    torch.cuda.synchronize()
                    ns = lat.cpu().numpy()
                elif mode == "invoke":
                    ctx.ce_pingpong(peer, initiator, size, iters, warmup, SRC_OFF, dst_off, FLAG_OFF, lat, status,
                                    int(timeout_s * 1e9))
                    torch.cuda.synchronize()
                    ns = lat.cpu().numpy()
                else:
                    ns = np.asarray(heap.native.host_ce_pingpong(peer, initiator, size, iters, warmup, SRC_OFF,
                                                                 dst_off, FLAG_OFF, timeout_s), dtype=np.int64)
                    torch.cuda.synchronize()
                if int(status[0].item()) != 0:
                    raise RuntimeError(f"{mode} ping-pong failed at {size} B: status {status.tolist()}")
                kdist.barrier()
                # the destination must hold the peer's source bytes (both directions were copied)
                mine = int(heap.tensor(dst_off, [size], torch.uint8).long().sum().item())
                theirs = int(src[:size].long().sum().item())
                sums = kdist.all_gather_objects((mine, theirs))
                ok = sums[0][0] == sums[1][1] and sums[1][0] == sums[0][1]
                one_way = float(np.percentile(ns, 50)) / 2 / 1e3 if initiator and len(ns) else 0.0
                row[f"{mode}_oneway_us"] = kdist.max_over_ranks(one_way)
                row[f"{mode}_ok"] = ok
            rows.append(row)
    finally:
        ctx.join_proxy_threads()
        del ctx
        del heap
    return rows


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--max-bytes", type=int, default=16 << 20)
    ap.add_argument("--iters", type=int, default=50)
    args = ap.parse_args()
    rank, world = kdist.init()
    sizes = [1 << i for i in range(3, int(np.log2(args.max_bytes)) + 1, 2)]
    rows = run(sizes, args.iters)
    if rank == 0:
        for r in rows:
            print("RESULT " + json.dumps({"bench": "ce_pingpong", **r}), flush=True)
    torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
