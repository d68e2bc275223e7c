"""EP transport benchmark: KiwiEpOp dispatch / combine captured in CUDA graphs.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 benchmarks/bench_ep_transport.py \\
        [--hidden 7168] [--tokens 128] [--experts-per-rank 32] [--topk 8] [--dtype bf16|fp8] [--iters 50]

The reference's transport benchmark (apps/ep/benchmarks/python/bench_kiwi_ep.py
of AMDResearch/kiwi: MORI-style op, graph-captured dispatch and combine, per
phase microseconds and GB/s from slot strides, :402-446) on this repository's
KiwiEpOp.  Three graphs are captured after an eager warm-up: dispatch alone,
combine alone (the received rows sent straight back), and one full round
(dispatch then combine).  The full round is replayed `iters` times between
barriers; dispatch and combine are replayed alternately (each dispatch epoch is
closed by its combine) with CUDA events around each replay, so their times
include waiting for the slowest peer.  Every reported time is the max over
ranks.  Bytes per rank: received tokens x the dispatch slot stride (row,
scales and metadata as stored) and received tokens x the bf16 row for combine.
Routing: `topk` distinct experts per token drawn uniformly (randperm), random
bf16 rows.  Prints one RESULT JSON line from rank 0.

Status: written against the same KiwiEpOp calls that tests/test_ep_gpu.py
exercises eagerly; the graph-captured runs have not been timed on a B200 yet.
"""
import argparse
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import torch  # noqa: E402

from kiwi_b200.parallel.ep import KiwiEpOp  # noqa: E402
from kiwi_b200.parallel.ep_collective import CollectiveEpOp  # noqa: E402
from kiwi_b200.utils import dist as kdist  # noqa: E402


def random_topk(tokens, experts, topk, gen, device):
    idx = torch.stack([torch.randperm(experts, generator=gen)[:topk] for _ in range(tokens)]).to(torch.int32)
    w = torch.rand(tokens, topk, generator=gen)
    return idx.to(device), (w / w.sum(-1, keepdim=True)).to(device)


def time_graph(g, iters):
    kdist.barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        g.replay()
    e.record()
    torch.cuda.synchronize()
    kdist.barrier()
    return kdist.max_over_ranks(s.elapsed_time(e) * 1e3 / iters)


def eager_and_report(op, dispatch, combine, args, rank, world):
    """CollectiveEpOp: dispatch and combine timed eagerly, events around each call, max over ranks."""
    s_d, e_d = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_c, e_c = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d_ms = c_ms = 0.0
    kdist.barrier()
    torch.cuda.synchronize()
    for _ in range(args.iters):
        s_d.record()
        cnt = dispatch()[4]
        e_d.record()
        s_c.record()
        combine()
        e_c.record()
        torch.cuda.synchronize()
        d_ms += s_d.elapsed_time(e_d)
        c_ms += s_c.elapsed_time(e_c)
    res = {"dispatch_us": kdist.max_over_ranks(d_ms * 1e3 / args.iters),
           "combine_us": kdist.max_over_ranks(c_ms * 1e3 / args.iters)}
    if rank == 0:
        print("RESULT " + json.dumps({"bench": "ep_transport", "transport": "collective", "world": world,
                                      "dtype": args.dtype, "hidden": args.hidden, "tokens_per_rank": args.tokens,
                                      "experts_per_rank": args.experts_per_rank, "topk": args.topk,
                                      "iters": args.iters, "recv_tokens_rank0": int(cnt.item()), **res,
                                      "split_e2e_us": res["dispatch_us"] + res["combine_us"],
                                      "timing": "eager, CUDA events, max over ranks"}), flush=True)
    kdist.barrier()


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--hidden", type=int, default=7168)
    ap.add_argument("--tokens", type=int, default=128, help="tokens per rank")
    ap.add_argument("--experts-per-rank", type=int, default=32)
    ap.add_argument("--topk", type=int, default=8)
    ap.add_argument("--dtype", default="bf16", choices=("bf16", "fp8"))
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--transport", default="nvlink", choices=("nvlink", "collective"),
                    help="KiwiEpOp (NVLink stores, CUDA graphs) or CollectiveEpOp (NCCL all-to-all, timed eagerly: "
                         "it reads the exchanged counts on the host)")
    args = ap.parse_args()

    rank, world = kdist.init()
    dev = torch.device("cuda", torch.cuda.current_device())
    dtype = torch.bfloat16 if args.dtype == "bf16" else torch.float8_e4m3fn
    op_cls = KiwiEpOp if args.transport == "nvlink" else CollectiveEpOp
    op = op_cls(hidden_dim=args.hidden, topk=args.topk, num_experts_per_rank=args.experts_per_rank,
                max_num_inp_token_per_rank=args.tokens, dispatch_dtype=dtype)
    gen = torch.Generator().manual_seed(1234 + rank)
    experts = args.experts_per_rank * world
    idx, w = random_topk(args.tokens, experts, args.topk, gen, dev)
    x = torch.randn(args.tokens, args.hidden, generator=gen).to(dev, torch.bfloat16)
    rows_back = torch.zeros(op.max_num_tokens_to_recv(), args.hidden, dtype=torch.bfloat16, device=dev)
    out = torch.empty(args.tokens, args.hidden, dtype=torch.bfloat16, device=dev)

    def dispatch():
        return op.dispatch(x, w, None, idx)

    def combine():
        op.combine(rows_back, None, idx, out=out)

    for _ in range(args.warmup):  # eager rounds: every rank's kernels and the epoch protocol warmed up
        dispatch()
        combine()
    torch.cuda.synchronize()
    op.check()
    kdist.barrier()

    if args.transport == "collective":
        eager_and_report(op, dispatch, combine, args, rank, world)
        return

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graphs = {}
    with torch.cuda.stream(side):
        for name, fn in (("dispatch", dispatch), ("combine", combine),
                         ("e2e", lambda: (dispatch(), combine()))):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                fn()
            graphs[name] = g
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    kdist.barrier()

    # Replays alternate dispatch and combine so every dispatch epoch is closed by its combine.
    for _ in range(2):
        graphs["dispatch"].replay()
        graphs["combine"].replay()
    torch.cuda.synchronize()
    kdist.barrier()
    res = {"e2e_us": time_graph(graphs["e2e"], args.iters)}
    # dispatch and combine alternate (each dispatch epoch is closed by its
    # combine) with events around each replay.
    kdist.barrier()
    torch.cuda.synchronize()
    s_d, e_d = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_c, e_c = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d_ms = c_ms = 0.0
    for _ in range(args.iters):
        s_d.record()
        graphs["dispatch"].replay()
        e_d.record()
        s_c.record()
        graphs["combine"].replay()
        e_c.record()
        torch.cuda.synchronize()
        d_ms += s_d.elapsed_time(e_d)
        c_ms += s_c.elapsed_time(e_c)
    res["dispatch_us"] = kdist.max_over_ranks(d_ms * 1e3 / args.iters)
    res["combine_us"] = kdist.max_over_ranks(c_ms * 1e3 / args.iters)
    op.check()

    _, _, _, _, cnt = dispatch()  # one eager round for this rank's received-token count
    combine()
    torch.cuda.synchronize()
    recv = int(cnt.item())
    lay = op.layout
    dispatch_slot = lay["row_bytes"] + lay["scale_bytes"] + lay["meta_bytes"]
    combine_slot = args.hidden * 2
    d_bytes = recv * dispatch_slot
    c_bytes = recv * combine_slot

    def gbs(b, us):
        return b / (us * 1e-6) / 1e9 if us > 0 else 0.0

    out_d = {"bench": "ep_transport", "world": world, "dtype": args.dtype, "hidden": args.hidden,
             "tokens_per_rank": args.tokens, "experts_per_rank": args.experts_per_rank, "topk": args.topk,
             "iters": args.iters, "recv_tokens_rank0": recv, **res,
             "split_e2e_us": res["dispatch_us"] + res["combine_us"],
             "dispatch_GBps_rank0": gbs(d_bytes, res["dispatch_us"]),
             "combine_GBps_rank0": gbs(c_bytes, res["combine_us"]),
             "e2e_GBps_rank0": gbs(d_bytes + c_bytes, res["e2e_us"]),
             "timing": "CUDA graphs, CUDA events, max over ranks"}
    graphs.clear()
    if rank == 0:
        print("RESULT " + json.dumps(out_d), flush=True)
    kdist.barrier()


if __name__ == "__main__":
    main()
