"""Grouped BF16 GEMM: kiwi tcgen05 kernel vs torch._grouped_mm (cuBLAS/CUTLASS)
on the expert-FFN shapes of the EP benchmark, per rank.

    python benchmarks/bench_gemm.py

Shapes: GEMM1 (K=7168 -> N=2*2048, SwiGLU epilogue for kiwi) and GEMM2
(K=2048 -> N=7168) for 32 experts x 1024 rows (one rank of 8) and 256 experts
x 128 rows (one rank of 1).  TFLOP/s from CUDA events over 20 launches after
warm-up; weights (B) exceed L2 in every shape.
"""
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import torch  # noqa: E402

import kiwi_b200  # noqa: E402
from kiwi_b200.ops import block_weights  # noqa: E402


def timeit(fn, iters=20):
    for _ in range(min(3, iters)):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def trace_stats(plan, counts, out, swiglu, groups, rows, k, n, bk):
    """One launch with the kernel's pipeline trace of CTA 0 (GroupedArgs::trace:
    per k-block, when the MMA warp started / ended its wait for a full stage and
    when the TMA producer started / ended its wait for a free stage, SM cycles),
    reduced to per-k-block statistics."""
    import numpy as np

    kb = k // bk
    tiles = groups * (rows // 128) * (n // 256)
    cap = kb * ((tiles + 147) // 148)
    tr = torch.zeros(cap * 4, dtype=torch.int64, device="cuda")
    plan.run(counts, out, swiglu, None, 0, False, tr, bk)
    torch.cuda.synchronize()
    t = tr.view(-1, 4).cpu().numpy().astype(np.int64)
    t = t[t[:, 1] > 0]
    mma_wait = t[:, 1] - t[:, 0]
    prod_wait = t[:, 3] - t[:, 2]
    span = t[-1, 1] - t[0, 0]
    per_kb = np.diff(t[:, 1])
    issue = t[1:, 0] - t[:-1, 1]        # MMA warp: stage ready -> next wait (issue + commit)
    lat = (t[:, 1] - t[:, 3])[t[:, 3] > 0]  # producer issue -> stage full seen by the MMA warp
    pct = lambda a, q: float(np.percentile(a, q))  # noqa: E731
    return {"kblocks_traced": int(len(t)), "span_cycles": int(span),
            "cycles_per_kblock_p50": pct(per_kb, 50), "cycles_per_kblock_mean": float(per_kb.mean()),
            "ideal_cycles_per_kblock": 128 * 256 * bk * 2 / 8192,
            "mma_wait_full_p50": pct(mma_wait, 50), "mma_wait_full_p90": pct(mma_wait, 90),
            "mma_wait_full_frac": float(mma_wait.sum() / span), "mma_issue_p50": pct(issue, 50),
            "producer_wait_empty_frac": float(prod_wait.sum() / span),
            "issue_to_full_p10": pct(lat, 10), "issue_to_full_p50": pct(lat, 50), "issue_to_full_p90": pct(lat, 90)}


SHAPES = [
    ("gemm1_ep8", 32, 1024, 7168, 4096, True),
    ("gemm2_ep8", 32, 1024, 2048, 7168, False),
    ("gemm1_ep1", 256, 128, 7168, 4096, True),
    ("gemm2_ep1", 256, 128, 2048, 7168, False),
]


def main():
    import argparse

    ap = argparse.ArgumentParser()
    ap.add_argument("--shape", default=None, help="run one shape only (e.g. gemm1_ep8)")
    ap.add_argument("--groups", type=int, default=None, help="override the group count")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--no-torch", action="store_true")
    ap.add_argument("--no-pair", action="store_true", help="skip the 2-SM (cta_group::2) kernel")
    ap.add_argument("--trace", action="store_true",
                    help="after timing, run one launch with the kernel's pipeline trace of CTA 0 and print its "
                         "per-k-block statistics (1-SM kernel)")
    ap.add_argument("--bk", type=int, default=64, choices=(64, 32, 128),
                    help="K columns per pipeline stage of the 1-SM kernel (32: 64-byte swizzle, 9 stages; "
                         "128: two 64-column boxes per operand, 2 stages)")
    ap.add_argument("--blocked", action="store_true",
                    help="weights (B) in the blocked layout: one contiguous 256 x 64 box per TMA load")
    ap.add_argument("--no-m64", action="store_true",
                    help="1-SM kernel: M = 128 MMAs on every tile (default: M = 64 on tiles with <= 64 rows left)")
    args = ap.parse_args()
    C = kiwi_b200.native()
    torch.manual_seed(0)
    for name, groups, rows, k, n, swiglu in SHAPES:
        if args.shape and name != args.shape:
            continue
        groups = args.groups or groups
        total = groups * rows
        a = (torch.randn(total, k, device="cuda") * 0.5).bfloat16()
        b = (torch.randn(groups * n, k, device="cuda") * 0.02).bfloat16()
        counts = torch.full((groups,), rows, dtype=torch.int32, device="cuda")
        out = torch.empty(total, n // 2 if swiglu else n, device="cuda", dtype=torch.bfloat16)
        plan = C.ops.GroupedGemm(a, block_weights(b, groups) if args.blocked else b, groups,
                                 b_blocked=args.blocked)
        ms = timeit(lambda: plan.run(counts, out, swiglu, None, 0, False, None, args.bk, not args.no_m64),
                    args.iters)
        ms_pair = float("nan")
        if rows >= 256 and not args.no_pair:
            ms_pair = timeit(lambda: plan.run(counts, out, swiglu, None, 0, True), args.iters)
        flops = 2.0 * total * n * k
        bw = (b.numel() * 2 + a.numel() * 2 + out.numel() * 2) / (ms / 1e3) / 1e12
        offs = torch.cumsum(counts, 0).to(torch.int32)
        bt = b.view(groups, n, k).transpose(-2, -1)
        tms = float("nan")
        if not args.no_torch:
            try:
                tms = timeit(lambda: torch._grouped_mm(a, bt, offs=offs, out_dtype=torch.bfloat16), args.iters)
            except Exception as ex:  # pragma: no cover
                print("torch._grouped_mm failed:", ex, file=sys.stderr)
        if args.trace:
            print("RESULT " + json.dumps({"bench": name + "_trace", "bk": args.bk,
                                          **trace_stats(plan, counts, out, swiglu, groups, rows, k, n, args.bk)}),
                  flush=True)
        print("RESULT " + json.dumps({"bench": name, "groups": groups, "rows": rows, "k": k, "n": n, "bk": args.bk,
                                      "kiwi_ms": ms, "kiwi_tflops": flops / ms / 1e9,
                                      "kiwi_pair_ms": ms_pair, "kiwi_pair_tflops": flops / ms_pair / 1e9,
                                      "kiwi_hbm_TBps_min_traffic": bw,
                                      "torch_grouped_mm_ms": tms, "torch_tflops": flops / tms / 1e9}), flush=True)


if __name__ == "__main__":
    main()
