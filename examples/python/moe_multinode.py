"""An expert-parallel MoE layer whose ranks need not share a node: CollectiveMoE
(dispatch and combine over torch.distributed all-to-all, experts on the
grouped GEMM) checked against the fp32 layer reference on every rank.

    # two nodes of 8 GPUs (NCCL)
    torchrun --nnodes 2 --nproc-per-node 8 --rdzv-backend c10d --rdzv-endpoint HOST:PORT \\
        examples/python/moe_multinode.py
    # two CPU processes (gloo), no GPU needed
    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 examples/python/moe_multinode.py --cpu

Every rank runs --steps forward passes on its own synthetic tokens, compares
the output with ``kiwi_b200.models.moe.moe_reference`` and reports the largest
relative error; rank 0 prints one RESULT line with the max over ranks of the
error and of the per-step time (CUDA events on GPU, wall clock on CPU).
Within one node, ``kiwi_b200.parallel.ep.ExpertParallelMoE`` (NVLink stores,
fused GEMMs) is the faster layer; this one is for ranks it cannot reach.
"""
import argparse
import json
import os
import sys
import time

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
import torch  # noqa: E402

from kiwi_b200.models import moe  # noqa: E402
from kiwi_b200.parallel.ep_collective import CollectiveMoE  # noqa: E402
from kiwi_b200.utils import dist as kdist  # noqa: E402


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--cpu", action="store_true", help="gloo process group and CPU tensors")
    ap.add_argument("--hidden", type=int, default=1024)
    ap.add_argument("--ffn", type=int, default=512)
    ap.add_argument("--experts-per-rank", type=int, default=4)
    ap.add_argument("--topk", type=int, default=4)
    ap.add_argument("--tokens", type=int, default=128)
    ap.add_argument("--quant", default="fp8", choices=["none", "fp8"])
    ap.add_argument("--steps", type=int, default=3)
    args = ap.parse_args(argv)
    rank, world = kdist.init(backend="gloo" if args.cpu else None, timeout_s=120.0, device=not args.cpu)
    device = torch.device("cpu") if args.cpu else torch.device("cuda", torch.cuda.current_device())
    cfg = moe.MoEConfig(hidden=args.hidden, ffn=args.ffn, num_experts=args.experts_per_rank * world,
                        topk=args.topk, tokens_per_rank=args.tokens, quant=args.quant, name="multinode")
    layer = CollectiveMoE(cfg, device=device)
    worst, times = 0.0, []
    for step in range(args.steps):
        x, logits = moe.synthetic_inputs(cfg, rank, device, step=step)
        if device.type == "cuda":
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            out = layer(x, logits)
            e.record()
            torch.cuda.synchronize()
            layer.check()
            times.append(s.elapsed_time(e))
        else:
            t0 = time.perf_counter()
            out = layer(x, logits)
            times.append((time.perf_counter() - t0) * 1e3)
        idx, w = moe.route_reference(logits, cfg.topk)
        ref = moe.moe_reference(cfg, x, idx, w, device=device)
        worst = max(worst, (out.float() - ref).abs().max().item() / max(ref.abs().max().item(), 1e-6))
    err = kdist.max_over_ranks(worst)
    ms = kdist.max_over_ranks(min(times))
    ok = err <= 2e-2
    if rank == 0:
        print("RESULT " + json.dumps({"example": "moe_multinode", "world": world, "device": device.type,
                                      "quant": cfg.quant, "tokens_per_rank": cfg.tokens_per_rank,
                                      "max_rel_err": round(err, 5), "ok": ok, "ms_per_step": round(ms, 3)}),
              flush=True)
    if kdist.dist.is_initialized():
        kdist.dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
