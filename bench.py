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
final reduction.  Weak scaling: tokens per rank are fixed as N grows.  The
timed steps run one round at a time; --in-flight 2 keeps two rounds in flight
instead (each a full layer forward of its own 4096 tokens per rank on its own
buffers and stream, so one round's dispatch / receive / combine overlap the
other's GEMMs) and then also reports the one-at-a-time time as `serial`.

Timing: W warm-up steps, then K steps bracketed by a barrier and
torch.cuda.synchronize() on both sides, CUDA events on the launching stream,
max over ranks.  The per-step working set (expert weights: 22.5 GB at N=1,
2.8 GB per GPU at N=8) is far larger than the 126 MB L2, so every step starts
with cold weights.  `value` is the whole-job aggregate tokens/s.

Besides the headline layer, the same run measures (all untimed parts excluded
from `value`):
* `checked`: one untimed step compared with the fp32 reference layer on a
  sampled subset of every rank's tokens;
* `baseline`: the on-box NCCL all-to-all + torch._grouped_mm layer
  (kiwi_b200.parallel.baseline) at the same N, config, seeds, warm-up and
  steps; `vs_baseline` is value / baseline value;
* `nvfp4`: BASELINE config 5 (hidden 4096, 64 experts, top-6, 8192 tokens per
  rank, Zipf(1.2) routing, NVFP4 dispatch), fused layer and NCCL baseline;
* `invoke_rtt`: the GPU->CPU->GPU round trip (1 block x 64 threads, 8-byte
  payload, 1,000,000 iterations after 10,000 warm-up), a payload sweep
  8 B - 4 KB, and the raw PCIe store-and-poll floor of the same box.
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


# route, begin, dispatch, dispatch-flag wait, recv_count, 2 schedules, recv assign (+ copy without the GEMM1
# gather), GEMM1, GEMM2 (+ combine send when unfused), combine-flag wait, combine reduce
def kernels_per_step(fused, gather):
    return 12 + (0 if fused else 1) + (0 if gather else 1)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="kiwi", choices=["kiwi", "reference", "nccl"])
    ap.add_argument("--config", default="deepseek_fp8")
    ap.add_argument("--tokens", type=int, default=None, help="override tokens per rank")
    ap.add_argument("--latency-tokens", type=int, default=128)
    ap.add_argument("--invoke-iters", type=int, default=1_000_000)
    ap.add_argument("--invoke-warmup", type=int, default=10_000)
    ap.add_argument("--sweep-iters", type=int, default=100_000, help="iterations per payload size of the sweep")
    ap.add_argument("--check-tokens", type=int, default=16, help="tokens per rank the correctness check samples")
    ap.add_argument("--in-flight", type=int, default=1,
                    help="rounds of the fused layer in flight during the timed steps (1: one round at a time)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-baseline", action="store_true", help="skip the in-process NCCL baseline")
    ap.add_argument("--no-nvfp4", action="store_true", help="skip the NVFP4 (config 5) sub-record")
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


def time_steps(step, warmup, steps, clocks=None, finish=None):
    """Device ms per step of `step()`: warm-up, then `steps` steps between CUDA
    events on the current stream, barrier + synchronize on both sides, max
    over ranks.  `finish()` (steps submitted to other streams) orders their
    completion on the current stream before the end event."""
    from kiwi_b200.utils import dist as kdist

    for _ in range(warmup):
        step()
    if finish is not None:
        finish()
    torch.cuda.synchronize()
    if clocks is not None:
        clocks.wait_first_sample()
    kdist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if clocks is not None:
        clocks.mark_start()
    start.record()
    for _ in range(steps):
        step()
    if finish is not None:
        finish()
    end.record()
    torch.cuda.synchronize()
    if clocks is not None:
        clocks.mark_end()
    kdist.barrier()
    return kdist.max_over_ranks(start.elapsed_time(end) / steps)


def check_layer(layer, cfg, x, logits, rank, samples):
    """One untimed step; the outputs of `samples` seeded token picks of this
    rank against the fp32 reference layer.  Returns (all ranks ok, max
    relative error over ranks)."""
    from kiwi_b200.models import moe as moe_model
    from kiwi_b200.utils import dist as kdist

    out = layer(x, logits).float()
    torch.cuda.synchronize()
    if hasattr(layer, "check"):
        layer.check()
    g = torch.Generator(device="cpu").manual_seed(1234 + rank)
    pick = torch.randperm(x.shape[0], generator=g)[:samples].to(x.device)
    idx, w = moe_model.route_reference(logits[pick], cfg.topk)
    ref = moe_model.moe_reference(cfg, x[pick], idx, w, device=x.device)
    err = (out[pick] - ref).abs().max().item() / max(ref.abs().max().item(), 1e-6)
    tol = 5e-2 if cfg.quant == "nvfp4" else 2e-2
    worst = kdist.max_over_ranks(err)
    return worst <= tol, worst


def run_layer(impl, cfg, rank, world, dev, args, clocks=None, max_tokens=None, keep=False, in_flight=1):
    """Builds the `impl` layer of `cfg`, checks it and times it.  Returns
    (layer, x, logits, record) with keep=True, else only the record (the layer
    and its inputs are released first).  With in_flight > 1 (fused layer) the
    timed steps are submitted rounds, that many in flight; the serial time of
    the same layer (one round at a time) is measured too."""
    from kiwi_b200.models import moe as moe_model

    if impl == "kiwi":
        from kiwi_b200.parallel.ep import ExpertParallelMoE

        layer = ExpertParallelMoE(cfg, max_tokens=max_tokens or cfg.tokens_per_rank, in_flight=in_flight)
        layer.set_flags(fused_combine=not args.unfused_combine, gather_a=args.gather)
    else:
        from kiwi_b200.parallel.baseline import NcclMoEBaseline

        layer = NcclMoEBaseline(cfg)
        in_flight = 1
    x, logits = moe_model.synthetic_inputs(cfg, rank, dev)
    ok, err = check_layer(layer, cfg, x, logits, rank, args.check_tokens)
    T = cfg.tokens_per_rank
    serial = None
    if in_flight > 1:
        serial_ms = time_steps(lambda: layer(x, logits), args.warmup, args.steps)
        serial = {"ms_per_step": serial_ms, "value": world * T / (serial_ms / 1e3), "rounds_in_flight": 1}
        ms = time_steps(lambda: layer.submit(x, logits), args.warmup, args.steps, clocks, finish=layer.wait_all)
    else:
        ms = time_steps(lambda: layer(x, logits), args.warmup, args.steps, clocks)
    if impl == "kiwi":
        layer.check()
    rec = {"impl": impl, "value": world * T / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
           "rounds_in_flight": in_flight, "serial": serial,
           "checked": bool(ok), "check_max_rel_err": err, "check_tokens_per_rank": args.check_tokens,
           "tflops_per_gpu": cfg.flops_per_token() * T / (ms / 1e3) / 1e12}
    if keep:
        return layer, x, logits, rec
    del layer, x, logits
    _release()
    return rec


def _release():
    """Returns freed device memory to the driver between measurements."""
    import gc

    gc.collect()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


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

    clocks = ClockSampler(device_index=_physical_index())
    with clocks:
        layer, x, logits, main_rec = run_layer(args.impl, cfg, rank, world, dev, args, clocks,
                                               max_tokens=max(T, args.latency_tokens), keep=True,
                                               in_flight=args.in_flight)
    ms = main_rec["ms_per_step"]
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
        del pipe

    # ---- latency mode (128 tokens per rank) on the same layer ----
    lat = None
    if args.impl == "kiwi" and args.latency_tokens:
        xl, ll = moe_model.synthetic_inputs(cfg, rank, dev, tokens=args.latency_tokens)
        lat_ms = time_steps(lambda: layer(xl, ll), 3, args.steps)
        lat = {"tokens_per_rank": args.latency_tokens, "us_per_step": lat_ms * 1e3,
               "tokens_per_s": world * args.latency_tokens / (lat_ms / 1e3)}
    layer_fused = args.impl == "kiwi" and not args.unfused_combine
    del layer, x, logits
    _release()

    # ---- the on-box NCCL baseline at the same N, config, seeds and steps ----
    base = None
    if args.impl == "kiwi" and not args.no_baseline:
        base = run_layer("nccl", cfg, rank, world, dev, args)
        base["what"] = ("NCCL all_to_all_single (one packed record per token and destination rank, one all-to-all "
                        "each way after the row-count exchange) + torch._grouped_mm, same process, N, config, "
                        "seeds, warm-up and steps")

    # ---- NVFP4 dispatch, hidden 4096, 64 experts, top-6, 8192 tokens, Zipf(1.2) ----
    nvfp4 = None
    if args.impl == "kiwi" and not args.no_nvfp4 and args.config == "deepseek_fp8":
        c5 = moe_model.CONFIGS["nvfp4"]
        r5 = run_layer("kiwi", c5, rank, world, dev, args, in_flight=args.in_flight)
        nvfp4 = {"config": "hidden 4096, expert FFN 4096->1536->4096 SwiGLU, 64 experts top-6, NVFP4 dispatch, "
                           "8192 tokens per rank, Zipf(1.2) router skew", **r5}
        if not args.no_baseline:
            rb5 = run_layer("nccl", c5, rank, world, dev, args)
            nvfp4["baseline"] = rb5
            nvfp4["vs_baseline"] = r5["value"] / rb5["value"]

    # ---- GPU -> CPU -> GPU invoke round trip (rank 0's GPU) ----
    invoke = None
    if args.impl == "kiwi" and rank == 0 and args.invoke_iters:
        invoke = measure_invoke(args)
    kdist.barrier()

    if rank == 0:
        tokens_s = main_rec["value"]
        line = {
            "metric": METRIC, "value": tokens_s, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": (tokens_s / base["value"]) if base else None,
            "vs_baseline_basis": "on-box NCCL + torch._grouped_mm layer measured in this run (see baseline)"
            if base else None,
            "dtype": "bf16", "data": "synthetic (seeded N(0,1) tokens and router logits, "
            "N(0,0.02) random-init expert weights)",
            "config": {"model": f"MoE expert FFN {cfg.hidden}->{cfg.ffn}->{cfg.hidden} SwiGLU, "
                                f"{cfg.num_experts} experts top-{cfg.topk}, {cfg.quant} dispatch ({args.config})",
                       "global_batch": world * T, "seq_len": 1, "tokens_per_rank": T,
                       "parallelism": f"ep{world}", "l2": "working set per step > L2 (expert weights "
                       f"{cfg.num_experts // world * 3 * cfg.hidden * cfg.ffn * 2 / 1e9:.1f} GB per GPU)"},
            "rounds_in_flight": main_rec["rounds_in_flight"], "serial": main_rec["serial"],
            "checked": main_rec["checked"], "check_max_rel_err": main_rec["check_max_rel_err"],
            "dispatch_combine_us": ms * 1e3,
            "tflops_per_gpu": main_rec["tflops_per_gpu"],
            "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"], "reasons": clk["reasons"],
                       "samples": clk["samples"]},
            "e2e": e2e, "gpu_launches": kernels_per_step(not args.unfused_combine, args.gather) * args.steps
            if args.impl == "kiwi" else None,
            "fused_combine": layer_fused if args.impl == "kiwi" else None,
            "gather_a": args.gather if args.impl == "kiwi" else None,
            "latency_mode": lat, "baseline": base, "nvfp4": nvfp4, "invoke_rtt": invoke, "impl": args.impl,
        }
        emit(line)
    if torch.distributed.is_initialized():
        torch.distributed.destroy_process_group()


def measure_invoke(args):
    """one persistent block of 64 threads enqueues an 8-byte
    seeded payload, a host callback increments it and replies through the
    mailbox, the kernel polls; iterations after warm-up; then the payload sweep
    (ring replies) and the raw PCIe store-and-poll floor of this box."""
    import numpy as np

    import kiwi_b200

    C = kiwi_b200.native()

    def stats(r):
        cyc = np.asarray(r["lat_cycles"], dtype=np.float64) * r["total_ns"] / max(r["total_cycles"], 1)
        return float(np.percentile(cyc, 50)) / 1e3, float(np.percentile(cyc, 99)) / 1e3

    r = C.bench.invoke_rtt(iters=args.invoke_iters, warmup=args.invoke_warmup, payload_bytes=8, mailbox=True,
                           block_threads=64)
    p50, p99 = stats(r)
    sweep = []
    for b in (8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096):
        rs = C.bench.invoke_rtt(iters=args.sweep_iters, warmup=max(1000, args.invoke_warmup // 10), payload_bytes=b,
                                mailbox=False, poll_warps=1, block_threads=64)
        s50, s99 = stats(rs)
        sweep.append({"payload_bytes": b, "ok": bool(rs["ok"]), "p50_us": s50, "p99_us": s99})
    fl = C.bench.pcie_floor(args.sweep_iters, max(1000, args.invoke_warmup // 10), -1)
    f50, f99 = stats(fl)
    return {"ok": bool(r["ok"]) and all(s["ok"] for s in sweep) and bool(fl["ok"]), "p50_us": p50, "p99_us": p99,
            "iters": args.invoke_iters, "warmup": args.invoke_warmup, "block": "1 x 64 threads",
            "payload_bytes": 8, "reply": "mailbox", "vs_baseline": BASELINE_INVOKE_P50_US / p50,
            "pcie_floor": {"p50_us": f50, "p99_us": f99, "iters": args.sweep_iters},
            "payload_sweep": sweep}


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
