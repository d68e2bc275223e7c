"""Headline benchmark: expert-parallel MoE dispatch+combine layer on B200, plus
the GPU->CPU->GPU invoke round trip.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl kiwi|reference|nccl]
    torchrun --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

Config (the headline MoE EP benchmark, throughput mode): hidden 7168, expert FFN
7168 -> 2048 -> 7168 SwiGLU (bf16 compute, fp32 accumulate), 256 experts sharded
evenly over the N GPUs, top-8 routing (softmax over the top-k) from N(0,1)
router logits, 4096 tokens per rank of N(0,1) bf16 activations, 1x128
block-scaled FP8 e4m3 dispatch, random-init N(0,0.02) weights, seeded
synthetic data.  A step is one full layer forward: routing, FP8 dispatch over
NVLink, expert-major layout, two grouped GEMMs, combine over NVLink and the
final reduction.  Weak scaling: tokens per rank are fixed as N grows.

Timing: W warm-up steps, then K steps bracketed by a barrier and
torch.cuda.synchronize() on both sides, CUDA events on the launching stream,
max over ranks.  The per-step working set (expert weights: 22.5 GB at N=1,
2.8 GB per GPU at N=8) is far larger than the 126 MB L2, so every step starts
with cold weights.  `value` is the whole-job aggregate tokens/s.
"""
import argparse
import json
import os
import sys

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "p50 GPU→CPU→GPU invoke µs; EP dispatch+combine µs & tokens/s at 1/2/4/8 B200"
BASELINE_INVOKE_P50_US = 1.92   # published reference number (MI300X)
# route, begin, dispatch, recv_count, 2 schedules, recv assign (+ copy without the GEMM1 gather), GEMM1,
# GEMM2 (+ combine send when unfused), combine reduce
def kernels_per_step(fused, gather):
    return 10 + (0 if fused else 1) + (0 if gather else 1)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="kiwi", choices=["kiwi", "reference", "nccl"])
    ap.add_argument("--config", default="deepseek_fp8")
    ap.add_argument("--tokens", type=int, default=None, help="override tokens per rank")
    ap.add_argument("--latency-tokens", type=int, default=128)
    ap.add_argument("--invoke-iters", type=int, default=200000)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--gather", action="store_true",
                    help="GEMM1 gathers its A rows from the receive slots (opt-in, comparison only)")
    ap.add_argument("--unfused-combine", action="store_true",
                    help="GEMM2 to local memory + combine send/receive kernels (comparison only)")
    return ap.parse_args()


def emit(obj):
    print(json.dumps(obj), flush=True)


def reference_unavailable(args):
    emit({"impl": "reference", "unavailable": "AMDResearch/kiwi is ROCm/HIP-only (gfx90a/942/950, CMake + HIP, "
          "no setup.py/pyproject; pip install of the reference checkout fails: not installable) and has no CUDA path "
          "to run on B200", "metric": METRIC, "n_gpus": args.gpus})


def main():
    args = parse()
    if args.impl == "reference":
        reference_unavailable(args)
        return
    from kiwi_b200.models import moe as moe_model
    from kiwi_b200.utils import dist as kdist
    from kiwi_b200.utils.clocks import ClockSampler
    from kiwi_b200.utils.pipeline import HostDevicePipeline
    from kiwi_b200.utils.topology import bind_process_to_gpu

    rank, world = kdist.init()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    dev = torch.device("cuda", torch.cuda.current_device())
    # Host buffers and threads on the GPU's NUMA node (pinned pages are placed
    # on the allocating thread's node).
    bind_process_to_gpu(dev.index)
    cfg = moe_model.CONFIGS[args.config]
    if args.tokens:
        cfg = moe_model.MoEConfig(**{**cfg.__dict__, "tokens_per_rank": args.tokens})
    T = cfg.tokens_per_rank

    if args.impl == "kiwi":
        from kiwi_b200.parallel.ep import ExpertParallelMoE

        layer = ExpertParallelMoE(cfg, max_tokens=max(T, args.latency_tokens))
        layer.native.fused_combine = not args.unfused_combine
        layer.native.gather_a = args.gather
    else:
        from kiwi_b200.parallel.baseline import NcclMoEBaseline

        layer = NcclMoEBaseline(cfg)
    x, logits = moe_model.synthetic_inputs(cfg, rank, dev)

    def step(xx, ll):
        return layer(xx, ll)

    clocks = ClockSampler(device_index=_physical_index())
    with clocks:
        for _ in range(args.warmup):
            step(x, logits)
        torch.cuda.synchronize()
        if args.impl == "kiwi":
            layer.check()
        clocks.wait_first_sample()

        # ---- timed region: K device-timed steps ----
        kdist.barrier()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clocks.mark_start()
        start.record()
        for _ in range(args.steps):
            step(x, logits)
        end.record()
        torch.cuda.synchronize()
        clocks.mark_end()
    kdist.barrier()
    ms = kdist.max_over_ranks(start.elapsed_time(end) / args.steps)
    if args.impl == "kiwi":
        layer.check()
    clk = clocks.summary()

    # ---- end to end through the public API: every step copies its inputs from
    # pinned host memory and its result back to pinned host memory; the copies of
    # neighbouring steps overlap the compute (HostDevicePipeline, 2 slots). ----
    e2e = None
    if not args.no_e2e:
        x_h = x.cpu().pin_memory()
        l_h = logits.cpu().pin_memory()
        out_h = [torch.empty(T, cfg.hidden, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
        if args.impl == "kiwi":
            def fn(xx, ll, out):
                layer(xx, ll, out=out)
        else:
            def fn(xx, ll, out):
                out.copy_(layer(xx, ll))
        pipe = HostDevicePipeline(fn, [(tuple(x.shape), x.dtype), (tuple(logits.shape), logits.dtype)],
                                  ((T, cfg.hidden), torch.bfloat16), depth=2)
        pipe.run(3, lambda i: (x_h, l_h), lambda i: out_h[i % 2], timed=False)
        torch.cuda.synchronize()
        kdist.barrier()
        torch.cuda.synchronize()
        e2e_ms = pipe.run(args.steps, lambda i: (x_h, l_h), lambda i: out_h[i % 2]) / args.steps
        torch.cuda.synchronize()
        kdist.barrier()
        e2e_ms = kdist.max_over_ranks(e2e_ms)
        e2e = {"value": world * T / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": x.numel() * x.element_size() + logits.numel() * logits.element_size(),
               "d2h_bytes_per_step": T * cfg.hidden * 2,
               "api": "kiwi_b200.utils.pipeline.HostDevicePipeline over ExpertParallelMoE.forward"
               if args.impl == "kiwi" else "HostDevicePipeline over NcclMoEBaseline.forward"}

    # ---- latency mode (128 tokens per rank) on the same layer ----
    lat = None
    if args.impl == "kiwi" and args.latency_tokens:
        xl, ll = moe_model.synthetic_inputs(cfg, rank, dev, tokens=args.latency_tokens)
        for _ in range(3):
            step(xl, ll)
        kdist.barrier()
        torch.cuda.synchronize()
        s3, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s3.record()
        for _ in range(args.steps):
            step(xl, ll)
        e3.record()
        torch.cuda.synchronize()
        kdist.barrier()
        lat_ms = kdist.max_over_ranks(s3.elapsed_time(e3) / args.steps)
        lat = {"tokens_per_rank": args.latency_tokens, "us_per_step": lat_ms * 1e3,
               "tokens_per_s": world * args.latency_tokens / (lat_ms / 1e3)}

    # ---- GPU -> CPU -> GPU invoke round trip (rank 0's GPU) ----
    invoke = None
    if args.impl == "kiwi" and rank == 0 and args.invoke_iters:
        import numpy as np

        import kiwi_b200

        r = kiwi_b200.native().bench.invoke_rtt(iters=args.invoke_iters, warmup=10000, payload_bytes=8,
                                                mailbox=True)
        cyc = np.asarray(r["lat_cycles"], dtype=np.float64) * r["total_ns"] / max(r["total_cycles"], 1)
        invoke = {"ok": bool(r["ok"]), "p50_us": float(np.percentile(cyc, 50)) / 1e3,
                  "p99_us": float(np.percentile(cyc, 99)) / 1e3, "iters": args.invoke_iters,
                  "vs_baseline": BASELINE_INVOKE_P50_US / (float(np.percentile(cyc, 50)) / 1e3)}
    kdist.barrier()

    if rank == 0:
        tokens_s = world * T / (ms / 1e3)
        flops = cfg.flops_per_token() * T  # per rank per step
        line = {
            "metric": METRIC, "value": tokens_s, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) tokens and router logits, "
            "N(0,0.02) random-init expert weights)",
            "config": {"model": f"MoE expert FFN {cfg.hidden}->{cfg.ffn}->{cfg.hidden} SwiGLU, "
                                f"{cfg.num_experts} experts top-{cfg.topk}, {cfg.quant} dispatch ({args.config})",
                       "global_batch": world * T, "seq_len": 1, "tokens_per_rank": T,
                       "parallelism": f"ep{world}", "l2": "working set per step > L2 (expert weights "
                       f"{cfg.num_experts // world * 3 * cfg.hidden * cfg.ffn * 2 / 1e9:.1f} GB per GPU)"},
            "dispatch_combine_us": ms * 1e3,
            "tflops_per_gpu": flops / (ms / 1e3) / 1e12,
            "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"], "reasons": clk["reasons"],
                       "samples": clk["samples"]},
            "e2e": e2e, "gpu_launches": kernels_per_step(not args.unfused_combine, args.gather) * args.steps
            if args.impl == "kiwi" else None,
            "fused_combine": (not args.unfused_combine) if args.impl == "kiwi" else None,
            "gather_a": args.gather if args.impl == "kiwi" else None,
            "latency_mode": lat, "invoke_rtt": invoke, "impl": args.impl,
        }
        emit(line)
    if torch.distributed.is_initialized():
        torch.distributed.destroy_process_group()


def _physical_index():
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    idx = torch.cuda.current_device()
    if vis:
        parts = [p.strip() for p in vis.split(",") if p.strip()]
        if idx < len(parts) and parts[idx].isdigit():
            return int(parts[idx])
    return idx


if __name__ == "__main__":
    main()
