"""GPU -> CPU -> GPU invoke round trip (one persistent block, 8-byte payload, payload sweep) and the raw PCIe floor.

    python benchmarks/bench_invoke.py [--iters 1000000] [--warmup 10000] [--sweep]

Prints one JSON ``RESULT`` line per configuration: p50/p99/mean microseconds
from %globaltimer deltas, and the same from %clock64 cycles scaled by the run's
measured ns/cycle (immune to the globaltimer's update granularity).
Reference: benchmarks/invoke/bench_latency.hip.cpp of AMDResearch/kiwi;
published bar 1.92 us p50 (MI300X).
"""
import argparse
import json
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import kiwi_b200  # noqa: E402


def summarize(name, r, extra=None):
    ns = np.asarray(r["lat_ns"], dtype=np.float64)
    cyc = np.asarray(r["lat_cycles"], dtype=np.float64)
    ns_per_cyc = r["total_ns"] / max(r["total_cycles"], 1)
    cyc_ns = cyc * ns_per_cyc
    out = {
        "bench": name,
        "ok": bool(r["ok"]),
        "iters": int(len(ns)),
        "p50_us": float(np.percentile(ns, 50)) / 1e3,
        "p99_us": float(np.percentile(ns, 99)) / 1e3,
        "mean_us": float(ns.mean()) / 1e3,
        "p50_us_cycles": float(np.percentile(cyc_ns, 50)) / 1e3,
        "p99_us_cycles": float(np.percentile(cyc_ns, 99)) / 1e3,
        "mean_us_total": r["total_ns"] / max(len(ns), 1) / 1e3,
        "sm_mhz_effective": 1e3 / ns_per_cyc if ns_per_cyc else None,
        "timer_distinct_values": int(len(np.unique(ns[: min(len(ns), 10000)]))),
    }
    if extra:
        out.update(extra)
    print("RESULT " + json.dumps(out), flush=True)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=1_000_000)
    ap.add_argument("--warmup", type=int, default=10_000)
    ap.add_argument("--sweep", action="store_true", help="payload sweep 8 B .. 4 KB")
    ap.add_argument("--poll-warps", type=int, nargs="*", default=[0, 2])
    ap.add_argument("--stagger", type=int, nargs="*", default=[100, 150, 200],
                    help="two-reads-in-flight mailbox mode: delay between the two reads (ns)")
    ap.add_argument("--cpu", type=int, default=-1)
    args = ap.parse_args()
    C = kiwi_b200.native()
    summarize("pcie_floor", C.bench.pcie_floor(args.iters, args.warmup, args.cpu))
    # Mailbox replies: one adaptive read in flight (the default), then two reads in flight a stagger apart.
    r = C.bench.invoke_rtt(iters=args.iters, warmup=args.warmup, cpu=args.cpu, mailbox=True, pipeline=1)
    summarize("invoke_rtt", r, {"payload_bytes": 8, "reply": "mailbox", "pipeline": 1, "queue": "spsc"})
    for st in args.stagger:
        r = C.bench.invoke_rtt(iters=args.iters, warmup=args.warmup, cpu=args.cpu, mailbox=True, pipeline=2,
                               stagger_ns=st)
        summarize("invoke_rtt", r, {"payload_bytes": 8, "reply": "mailbox", "pipeline": 2, "stagger_ns": st,
                                    "queue": "spsc"})
    for pw in args.poll_warps:
        r = C.bench.invoke_rtt(args.iters // 4, args.warmup, 8, 1, args.cpu, 4096, False, pw)
        summarize("invoke_rtt", r, {"payload_bytes": 8, "reply": "ring", "poll_warps": pw, "queue": "spsc"})
    r = C.bench.invoke_rtt(args.iters // 4, args.warmup, 8, 1, args.cpu, 4096, True, 0, 2_000_000_000, True, 200)
    summarize("invoke_rtt", r, {"payload_bytes": 8, "reply": "mailbox", "stagger_ns": 200, "queue": "mpsc"})
    # Host-mapped grid polling (reference: benchmarks/hardware/bench_host_mapped_grid_poll): block 0 publishes
    # through host memory, the other blocks' warps poll it, then ack back.
    sms = C.ops.num_sms()
    for blocks in (2, 16, min(64, sms), sms):
        g = C.bench.grid_poll(blocks=blocks, threads=256, rounds=2000, delay_ns=10_000)
        print("RESULT " + json.dumps({"bench": "grid_poll", "threads": 256, **g}), flush=True)
    # Device-side overhead of one invoke (reference: benchmarks/invoke/bench_overhead): SM cycles per call.
    for lm in (False, True):
        c = C.bench.invoke_cost(calls=100_000, lane_masked=lm)
        print("RESULT " + json.dumps({"bench": "invoke_cost", "lane_masked": lm, "args_bytes": 16,
                                      "messages_per_call": 16 if lm else 1, **c}), flush=True)
    for b in (8, 64, 256):
        c = C.bench.push_cost(msgs=100_000, payload_bytes=b)
        print("RESULT " + json.dumps({"bench": "push_cost", "payload_bytes": b, **c}), flush=True)
    if args.sweep:
        for b in [8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096]:
            r = C.bench.invoke_rtt(max(args.iters // 20, 1000), args.warmup // 10, b, 1, args.cpu, 4096, False,
                                   2)
            summarize("invoke_rtt_sweep", r, {"payload_bytes": b, "reply": "ring", "poll_warps": 2})


if __name__ == "__main__":
    main()
