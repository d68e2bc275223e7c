"""Copy bandwidth of the EP row patterns against the measured HBM copy peak.

    python benchmarks/bench_ep_copy.py [--hidden 7168] [--rows 16384] [--topk 8] [--iters 20] [--warmup 3]

Patterns, each on bf16 rows of `hidden` elements, with the native kernel
(``kiwi_b200.ops.copy_rows`` / ``accumulate_rows``) and the PyTorch op that
does the same:

    copy        dst[i] = src[i]                      (torch: dst.copy_(src))
    pack        dst[i] = src[perm[i]]                (torch: index_select(out=))
    unpack      dst[perm[i]] = src[i]                (torch: index_copy_)
    accumulate  out[t] = sum_j src[map[t, j]]         (torch: index_select + sum)
                with `topk` rows per token, every source row used once

With the defaults every pattern reads 235 MB (more than the 126 MB L2), so
back-to-back iterations stream from HBM.  Each RESULT line gives the
algorithmic bytes (rows read + rows written), GB/s from CUDA events, and the
fraction of the measured copy peak (``hbm_gbs`` of MEASURED_PEAKS.json at the
repository root; 6650 GB/s when that file is absent).  Counterpart of the
reference's apps/ep/benchmarks/bench_ep_copy.hip.cpp and
bench_ep_hidden_copy.hip.cpp of AMDResearch/kiwi.
"""
import argparse
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import torch  # noqa: E402

FALLBACK_HBM_GBS = 6650.0
PATTERNS = ("copy", "pack", "unpack", "accumulate")


def hbm_peak(path=os.path.join(ROOT, "MEASURED_PEAKS.json")):
    """(GB/s, source) of the copy roofline."""
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def algorithmic_bytes(pattern, rows, hidden, topk, elem=2):
    """Bytes a pattern must move: every row read once and every output row written once."""
    row = hidden * elem
    if pattern == "accumulate":
        return rows * row + (rows // topk) * row
    return 2 * rows * row


def build(pattern, rows, hidden, topk, device, seed=0):
    """(src, dst, index) of a pattern; index is int32 (perm [rows] or map [rows / topk, topk])."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    src = torch.randn(rows, hidden, generator=g).to(torch.bfloat16).to(device)
    perm = torch.randperm(rows, generator=g).to(torch.int32)
    if pattern == "accumulate":
        return src, torch.empty(rows // topk, hidden, dtype=torch.bfloat16, device=device), \
            perm[: rows // topk * topk].view(rows // topk, topk).to(device)
    return src, torch.empty(rows, hidden, dtype=torch.bfloat16, device=device), \
        (None if pattern == "copy" else perm.to(device))


def runner(pattern, impl, src, dst, index):
    """A no-argument callable doing one iteration of (pattern, impl)."""
    from kiwi_b200 import ops

    err = torch.zeros(1, dtype=torch.int32, device=src.device)
    if impl == "native":
        if pattern == "accumulate":
            return lambda: ops.accumulate_rows(src, index, dst, err), err
        si = index if pattern == "pack" else None
        di = index if pattern == "unpack" else None
        return lambda: ops.copy_rows(src, dst, si, di, None, err), err
    idx64 = None if index is None else index.long()
    if pattern == "copy":
        return lambda: dst.copy_(src), None
    if pattern == "pack":
        return lambda: torch.index_select(src, 0, idx64, out=dst), None
    if pattern == "unpack":
        return lambda: dst.index_copy_(0, idx64, src), None
    t, k = index.shape
    flat = idx64.view(-1)
    return lambda: dst.copy_(src.index_select(0, flat).view(t, k, -1).float().sum(1)), None


def agree(pattern, a, b):
    """Copies must match bit for bit; sums may differ in the order of fp32 additions."""
    if pattern != "accumulate":
        return torch.equal(a, b)
    return (a.float() - b.float()).abs().max().item() <= 1e-2 * b.float().abs().max().item()


def time_ms(fn, iters, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--hidden", type=int, default=7168)
    ap.add_argument("--rows", type=int, default=16384)
    ap.add_argument("--topk", type=int, default=8)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--patterns", default=",".join(PATTERNS))
    args = ap.parse_args(argv)
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    from kiwi_b200 import ops

    peak, peak_src = hbm_peak()
    dev = torch.device("cuda", torch.cuda.current_device())
    for pattern in [p for p in args.patterns.split(",") if p]:
        src, dst, index = build(pattern, args.rows, args.hidden, args.topk, dev)
        want = None
        for impl in ("native", "torch"):
            fn, err = runner(pattern, impl, src, dst, index)
            ms = time_ms(fn, args.iters, args.warmup)
            if err is not None:
                ops.check_error(err)
            if want is None:
                want = dst.clone()
            elif not agree(pattern, dst, want):
                raise RuntimeError(f"{pattern}: native and torch results differ")
            nbytes = algorithmic_bytes(pattern, args.rows, args.hidden, args.topk)
            gbs = nbytes / (ms * 1e-3) / 1e9
            print("RESULT " + json.dumps({
                "bench": "ep_copy", "pattern": pattern, "impl": impl, "rows": args.rows, "hidden": args.hidden,
                "topk": args.topk if pattern == "accumulate" else None, "bytes": nbytes, "ms": round(ms, 4),
                "gbs": round(gbs, 1), "frac_of_hbm": round(gbs / peak, 3), "hbm_peak": f"{peak} ({peak_src})",
                "l2": "inputs larger than L2"}), flush=True)
        del src, dst, index
    return 0


if __name__ == "__main__":
    sys.exit(main())
