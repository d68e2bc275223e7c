"""Single-GPU run of the P2P data-plane and collective kernels on a one-rank
heap (peer = this GPU), for profiling them in isolation: a 64 MB put with
release signal (the put_bw kernel, src and dst in this GPU's heap, rotating
over 256 MB) and 200 device all-to-all rounds.  Prints one RESULT line.

    python benchmarks/p2p_local_kernels.py
"""
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import torch  # noqa: E402

from kiwi_b200.parallel.collectives import DeviceCollectives  # noqa: E402
from kiwi_b200.parallel.p2p import SymmetricHeap  # noqa: E402
from kiwi_b200.utils import dist as kdist  # noqa: E402


def main():
    kdist.init()
    size, region = 64 << 20, 256 << 20
    heap = SymmetricHeap(4096 + 2 * region + 4096)
    src_off, dst_off = 4096, 4096 + region
    heap.tensor(src_off, [region], torch.uint8).copy_(torch.randint(0, 256, (region,), dtype=torch.uint8,
                                                                    device="cuda"))
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
    print("RESULT " + json.dumps({"bench": "p2p_local_kernels", "put_GBps_local": max(gbps),
                                  "all2all_round_us_world1": float(lat.float().median().item()) / 1e3}), flush=True)


if __name__ == "__main__":
    main()
