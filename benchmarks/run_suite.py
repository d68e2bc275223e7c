"""Run the benchmark suite and collect every RESULT line in one JSONL file.

    python benchmarks/run_suite.py [--gpus N] [--out results.jsonl] [--only invoke,gemm,...] [--quick] [--dry-run]

Single-GPU benchmarks run as plain processes; multi-rank ones run under
``torch.distributed.run`` on N GPUs of this node (127.0.0.1 rendezvous,
one process per GPU).  Each RESULT line is stored with the benchmark's name,
its command and the environment (``kiwi_b200.utils.env``); a benchmark that
fails is recorded with its exit status and the tail of its output, and the
suite continues.  A benchmark that runs past ``--timeout`` is ended with its
whole process group (torchrun and its ranks).  Counterpart of the reference's
sweep scripts (benchmarks/queue_baselines/run_sweep.sh, scripts/ep_bench/*.sh
of AMDResearch/kiwi).
"""
import argparse
import json
import os
import signal
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def suite(gpus, quick):
    """(name, multi_rank, argv) of every benchmark, smaller with `quick`."""
    def it(full, small):
        return small if quick else full

    return [
        ("queue", False, ["benchmarks/bench_queue.py"]),
        ("invoke", False, ["benchmarks/bench_invoke.py", "--iters", str(it(1_000_000, 20_000)),
                           "--warmup", str(it(10_000, 1_000))]),
        ("frontends", False, ["benchmarks/bench_frontends.py"]),
        ("gemm", False, ["benchmarks/bench_gemm.py"] + (["--shape", "gemm1_ep8", "--groups", "8"] if quick else [])),
        ("ep_copy", False, ["benchmarks/bench_ep_copy.py", "--iters", str(it(20, 5))]),
        ("p2p_local", False, ["benchmarks/bench_p2p.py", "--local"]),
        ("p2p", True, ["benchmarks/bench_p2p.py", "--iters", str(it(2000, 200))]),
        ("collectives", True, ["benchmarks/bench_collectives.py"]),
        ("ep_stages", True, ["benchmarks/bench_ep_stages.py", "--steps", str(it(10, 3))]),
        ("ep_transport", True, ["benchmarks/bench_ep_transport.py", "--iters", str(it(50, 10))]),
        ("ep_transport_collective", True, ["benchmarks/bench_ep_transport.py", "--transport", "collective",
                                           "--iters", str(it(50, 10))]),
        ("bench", True, ["bench.py", "--gpus", str(gpus), "--steps", str(it(40, 5)), "--warmup", str(it(5, 3))]),
    ]


def command(multi_rank, argv, gpus, port):
    """The command line of one benchmark (torchrun for multi-rank ones on more than one GPU)."""
    if multi_rank and gpus > 1:
        return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={gpus}",
                "--master-addr=127.0.0.1", f"--master-port={port}", *argv]
    return [sys.executable, *argv]


def run_group(cmd, timeout_s, grace_s=30):
    """Runs `cmd` in a session of its own; on timeout the whole process group
    it started (torchrun and its ranks) gets SIGTERM, then SIGKILL after
    `grace_s`.  Returns (exit status, or -1 on timeout, and the combined output)."""
    p = subprocess.Popen(cmd, cwd=ROOT, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True,
                         start_new_session=True)
    try:
        out, _ = p.communicate(timeout=timeout_s)
        return p.returncode, out
    except subprocess.TimeoutExpired:
        out = ""
        for sig, wait in ((signal.SIGTERM, grace_s), (signal.SIGKILL, 10)):
            try:
                os.killpg(p.pid, sig)
            except ProcessLookupError:
                break
            try:
                out, _ = p.communicate(timeout=wait)
                break
            except subprocess.TimeoutExpired:
                out = ""
        return -1, (out or "") + "\n[timed out]"


def parse_results(text):
    """The JSON objects a benchmark printed (RESULT lines and bare JSON lines)."""
    results = []
    for line in text.splitlines():
        line = line.strip()
        if line.startswith("RESULT "):
            line = line[len("RESULT "):]
        if line.startswith("{"):
            try:
                results.append(json.loads(line))
            except json.JSONDecodeError:
                pass
    return results


def main(argv=None):
    """Command-line entry; returns 0 when every benchmark exited 0."""
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1, help="GPUs for the multi-rank benchmarks")
    ap.add_argument("--out", default="suite_results.jsonl")
    ap.add_argument("--only", default="", help="comma-separated benchmark names (default: all)")
    ap.add_argument("--quick", action="store_true", help="small iteration counts (a smoke run of the suite)")
    ap.add_argument("--timeout", type=int, default=1800, help="seconds per benchmark")
    ap.add_argument("--port", type=int, default=29571)
    ap.add_argument("--dry-run", action="store_true", help="print the commands only")
    args = ap.parse_args(argv)
    only = {s for s in args.only.split(",") if s}
    all_entries = suite(args.gpus, args.quick)
    unknown = only - {e[0] for e in all_entries}
    if unknown:
        ap.error("unknown benchmark(s): " + ", ".join(sorted(unknown)))
    entries = [e for e in all_entries if not only or e[0] in only]
    if args.dry_run:
        for name, multi, av in entries:
            print(name + ": " + " ".join(command(multi, av, args.gpus, args.port)))
        return 0
    sys.path.insert(0, ROOT)
    from kiwi_b200.utils.env import collect_env

    env = collect_env()
    failures = 0
    with open(args.out, "a") as out:
        for name, multi, av in entries:
            cmd = command(multi, av, args.gpus, args.port)
            t0 = time.time()
            rc, text = run_group(cmd, args.timeout)
            rec = {"suite": name, "cmd": cmd, "exit": rc, "seconds": round(time.time() - t0, 1),
                   "results": parse_results(text), "env": env}
            if rc != 0:
                rec["tail"] = text[-3000:]
                failures += 1
            out.write(json.dumps(rec, default=str) + "\n")
            out.flush()
            print(f"{name}: exit {rc}, {len(rec['results'])} result(s), {rec['seconds']} s", flush=True)
    return 1 if failures else 0


if __name__ == "__main__":
    sys.exit(main())
