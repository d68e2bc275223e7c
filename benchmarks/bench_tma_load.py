"""What the TMA path feeds one SM, with every SM loading: the grouped GEMM's
operand pattern without its MMAs.

    python benchmarks/bench_tma_load.py [--iters 4000] [--json]

For box widths of 64 bf16 (128-byte rows, 128-byte swizzle) and 32 bf16
(64-byte rows, 64-byte swizzle), boxes of 128 and 256 rows, 2 to 8 stages, and
two sources: `stream` (each CTA walks rows of its own in a 940 MB tensor, as
the GEMM's activation tiles) and `l2` (every CTA walks the same rows, as the
weight tile that the m-tiles of one group share).  One CTA per SM; each CTA's
SM-cycle count comes from the kernel (`native().ops.tma_load_rate`), the
aggregate bandwidth from CUDA events around the launch.

Reading: the grouped GEMM needs 96 B/cycle/SM (a 48 KB stage per 512 MMA
cycles at 128 x 256 x 64) for the 1-SM tile and 64 B/cycle/SM for the 2-SM
tile; if rows/cycle stays flat while bytes/cycle halves from 128- to 64-byte
rows, the feed is bound by box rows rather than bytes.
"""
import argparse
import json
import os
import statistics
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import torch  # noqa: E402

import kiwi_b200  # noqa: E402


def run(ops, t, box_rows, box_k, stages, iters, shared):
    for _ in range(2):  # warm-up (tensor map, clocks)
        ops.tma_load_rate(t, box_rows, box_k, stages, max(64, iters // 16), 0, shared)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    cycles, err = ops.tma_load_rate(t, box_rows, box_k, stages, iters, 0, shared)
    e.record()
    torch.cuda.synchronize()
    if int(err.item()) != 0:
        raise RuntimeError(f"tma_load_rate: bounded wait ran out (code {int(err.item())})")
    cyc = [int(c) for c in cycles.tolist() if c > 0]
    med = statistics.median(cyc)
    box_bytes = box_rows * box_k * 2
    ms = s.elapsed_time(e)
    return {"box_rows": box_rows, "row_bytes": box_k * 2, "stages": stages, "source": "l2" if shared else "stream",
            "B_per_cycle_per_sm": box_bytes * iters / med, "rows_per_cycle_per_sm": box_rows * iters / med,
            "cycles_per_box": med / iters, "aggregate_TBps": box_bytes * iters * len(cyc) / (ms / 1e3) / 1e12,
            "ms": ms}


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--iters", type=int, default=4000, help="boxes per CTA")
    ap.add_argument("--rows", type=int, default=65536)
    ap.add_argument("--k", type=int, default=7168)
    args = ap.parse_args()
    ops = kiwi_b200.native().ops
    t = torch.randn(args.rows, args.k, device="cuda").bfloat16()
    for shared in (False, True):
        for box_k in (64, 32):
            for box_rows in (128, 256):
                for stages in (2, 4, 8):
                    if stages * box_rows * box_k * 2 + 2048 > 227 * 1024:
                        continue
                    r = run(ops, t, box_rows, box_k, stages, args.iters, shared)
                    print("RESULT " + json.dumps({"bench": "tma_load_rate", **r}), flush=True)


if __name__ == "__main__":
    main()
