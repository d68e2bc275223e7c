"""Device count all-to-all and barrier over NVLink vs NCCL (reference:
apps/ep/benchmarks/bench_ep_collectives.hip.cpp:234-250 of AMDResearch/kiwi,
which compares the GPU barrier / count all2all with the host library's).

    torchrun --nproc-per-node N --master-addr 127.0.0.1 benchmarks/bench_collectives.py

* kiwi_all2all_us: one round of the epoch-tagged u32 all-to-all (every rank
  stores into every peer's ingress cell and waits for all), p50 of the
  per-round device times of 2000 back-to-back rounds in one kernel.
* kiwi_barrier_us: the same for barrier rounds.
* nccl_all2all_us: torch.distributed.all_to_all_single of world int64 values,
  CUDA events over 200 calls.
* nccl_barrier_us: all_reduce of one int32 (NCCL's barrier), same timing.
Every number is the max over ranks.
"""
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from kiwi_b200.parallel.collectives import DeviceCollectives  # noqa: E402
from kiwi_b200.utils import dist as kdist  # noqa: E402


def timed(fn, iters):
    for _ in range(10):
        fn()
    torch.cuda.synchronize()
    kdist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters * 1e3


def main():
    rank, world = kdist.init()
    coll = DeviceCollectives()
    rounds = 2000
    send = torch.arange(world, dtype=torch.int32, device="cuda") + 1000 * rank
    out = torch.empty(rounds, world, dtype=torch.int32, device="cuda")
    lat = torch.zeros(rounds, dtype=torch.int64, device="cuda")
    coll.all2all(send, out=out, rounds=rounds, lat=lat)
    torch.cuda.synchronize()
    coll.check()
    a2a = float(np.percentile(lat.cpu().numpy()[100:], 50)) / 1e3
    ok = bool((out[-1].cpu() == torch.arange(world, dtype=torch.int32) * 1000 + rank + rounds - 1).all())
    coll.barrier(rounds=rounds, lat=lat)
    torch.cuda.synchronize()
    coll.check()
    bar = float(np.percentile(lat.cpu().numpy()[100:], 50)) / 1e3
    x = torch.arange(world, dtype=torch.int64, device="cuda")
    y = torch.empty_like(x)
    one = torch.ones(1, dtype=torch.int32, device="cuda")
    nccl_a2a = timed(lambda: dist.all_to_all_single(y, x), 200) if world > 1 else 0.0
    nccl_bar = timed(lambda: dist.all_reduce(one), 200) if world > 1 else 0.0
    row = {"bench": "collectives", "world": world, "ok": kdist.max_over_ranks(0.0 if ok else 1.0) == 0.0,
           "kiwi_all2all_us": kdist.max_over_ranks(a2a), "kiwi_barrier_us": kdist.max_over_ranks(bar),
           "nccl_all2all_us": kdist.max_over_ranks(nccl_a2a), "nccl_barrier_us": kdist.max_over_ranks(nccl_bar)}
    if rank == 0:
        print("RESULT " + json.dumps(row), flush=True)
    del coll
    if dist.is_initialized():
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
