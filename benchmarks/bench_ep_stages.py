"""Per-stage device time of the fused EP MoE layer (CUDA events, max over ranks).

    python benchmarks/bench_ep_stages.py [--config deepseek_fp8] [--tokens 4096] [--steps 10]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 benchmarks/bench_ep_stages.py ...

Stages: route, dispatch (+begin), receive (count, schedules, assign, copy;
no copy with --gather), gemm1 (gate/up + SwiGLU; with --gather its A rows are
gathered and dequantised from the receive slots), gemm2 (down projection; with the fused combine its
epilogue also stores the rows over NVLink), combine (fused: wait + top-k sum;
--unfused: send + reduce).  A stage that waits for other ranks includes their
skew.  Prints one RESULT JSON line.
"""
import argparse
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import torch  # noqa: E402

from kiwi_b200.models import moe as moe_model  # noqa: E402
from kiwi_b200.parallel.ep import ExpertParallelMoE  # noqa: E402
from kiwi_b200.utils import dist as kdist  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="deepseek_fp8")
    ap.add_argument("--tokens", type=int, default=None)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--experts", type=int, default=None, help="override the expert count (small profiling cases)")
    ap.add_argument("--unfused", action="store_true", help="GEMM2 to local memory + combine send/receive")
    ap.add_argument("--gather", action="store_true", help="GEMM1 gathers its A rows from the receive slots")
    ap.add_argument("--debug-timing", action="store_true",
                    help="after the timed loop, run one round with device phase timing and print every rank's "
                         "per-kernel spans (first block start to last warp end, flag waits)")
    args = ap.parse_args()
    rank, world = kdist.init()
    cfg = moe_model.CONFIGS[args.config]
    if args.tokens:
        cfg = moe_model.MoEConfig(**{**cfg.__dict__, "tokens_per_rank": args.tokens})
    if args.experts:
        cfg = moe_model.MoEConfig(**{**cfg.__dict__, "num_experts": args.experts})
    layer = ExpertParallelMoE(cfg)
    layer.native.fused_combine = not args.unfused
    layer.native.gather_a = args.gather
    x, logits = moe_model.synthetic_inputs(cfg, rank, "cuda")
    out = torch.empty_like(x)
    names = ["route", "dispatch", "receive", "gemm1", "gemm2", "combine"]
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(names) + 1)]
    acc = [0.0] * len(names)
    for it in range(args.steps + 3):
        kdist.barrier()
        torch.cuda.synchronize()
        ev[0].record()
        idx, w = layer.route(logits)
        ev[1].record()
        layer.stage_dispatch(x, idx, w)
        ev[2].record()
        layer.stage_receive()
        ev[3].record()
        layer.native.experts_gemm(1)
        ev[4].record()
        layer.native.experts_gemm(2)
        ev[5].record()
        layer.stage_combine(idx, out)
        ev[6].record()
        torch.cuda.synchronize()
        if it >= 3:
            for i in range(len(names)):
                acc[i] += ev[i].elapsed_time(ev[i + 1])
    layer.check()
    if args.debug_timing:
        # Outside the timed loop: one more round with the stamps on.
        from kiwi_b200.parallel.ep import format_debug_timing

        layer.set_debug_timing_enabled(True)
        kdist.barrier()
        layer(x, logits, out)
        snap = layer.get_debug_timing_snapshot()
        layer.set_debug_timing_enabled(False)
        for r in range(world):
            if r == rank:
                print(format_debug_timing(snap, f"ep-{args.config}"), flush=True)
            kdist.barrier()
    res = {n: kdist.max_over_ranks(a / args.steps * 1e3) for n, a in zip(names, acc)}
    counts = layer.expert_counts.float()
    if rank == 0:
        print("RESULT " + json.dumps({"bench": "ep_stages_us", "config": args.config, "world": world,
                                      "fused_combine": not args.unfused, "gather_a": args.gather,
                                      "tokens_per_rank": cfg.tokens_per_rank, **res,
                                      "total_us": sum(res.values()),
                                      "rows_per_expert_mean": float(counts.mean()),
                                      "rows_per_expert_max": float(counts.max())}), flush=True)


if __name__ == "__main__":
    main()
