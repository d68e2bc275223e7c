"""Installation check: ``python -m kiwi_b200 [--smoke] [--json]``.

Reports whether the native extension loads, what it was built for, the
environment (``kiwi_b200.utils.env``), and, per visible GPU, whether it is an
sm_100 part, which peers it reaches over P2P and whether NVLS multicast is
available.  ``--smoke`` also runs the tiny end-to-end pass the test suite's
smoke check uses (a device-to-host queue round and one expert-parallel MoE
layer forward on cuda:0 against the fp32 reference) and an invoke round trip.
Counterpart of the reference's smoke-correctness gate
(scripts/ep_bench/run_kiwi_ep_smoke_correctness.sh of AMDResearch/kiwi).
Exit status 0 when every requested check passes.
"""
import argparse
import json
import sys


def gpu_checks(C):
    """Per visible GPU: generation, SMs, memory, P2P peers, NVLS support."""
    import torch

    out = []
    if not torch.cuda.is_available():
        return out
    n = torch.cuda.device_count()
    for i in range(n):
        p = torch.cuda.get_device_properties(i)
        g = {"index": i, "name": p.name, "capability": f"{p.major}.{p.minor}", "sm_100": (p.major, p.minor) == (10, 0),
             "sms": p.multi_processor_count, "memory_gib": round(p.total_memory / 2**30, 1),
             "p2p_peers": [j for j in range(n) if j != i and torch.cuda.can_device_access_peer(i, j)]}
        try:
            g["multicast"] = bool(C.p2p.multicast_supported(i))
        except Exception as e:  # noqa: BLE001 - report, do not fail the listing
            g["multicast"] = f"unknown ({e})"
        out.append(g)
    return out


def main(argv=None):
    """Command-line entry; returns the exit status."""
    ap = argparse.ArgumentParser(prog="python -m kiwi_b200", description=__doc__.splitlines()[0])
    ap.add_argument("--smoke", action="store_true", help="run the end-to-end smoke pass on cuda:0")
    ap.add_argument("--json", action="store_true", help="print one JSON document instead of text")
    args = ap.parse_args(argv)

    import kiwi_b200
    from kiwi_b200.utils import env

    report = {"version": kiwi_b200.__version__, "ok": True}
    try:
        C = kiwi_b200.native()
        report["extension"] = {"loaded": True, "file": getattr(C, "__file__", None)}
    except ImportError as e:
        report["extension"] = {"loaded": False, "error": str(e)}
        report["ok"] = False
        C = None
    report["env"] = env.collect_env()
    report["gpus"] = gpu_checks(C) if C is not None else []
    if report["gpus"] and not all(g["sm_100"] for g in report["gpus"]):
        report["warning"] = "kernels are built for sm_100a (B200); other GPUs cannot run them"
    if args.smoke:
        smoke = {}
        if C is None or not report["gpus"]:
            smoke["skipped"] = "needs the extension and a CUDA device"
            report["ok"] = False
        else:
            try:
                import torch

                from kiwi_b200 import smoke as _smoke

                torch.cuda.set_device(0)
                r = C.bench.invoke_rtt(iters=1000, warmup=100, payload_bytes=8)
                smoke["invoke_rtt_ok"] = bool(r["ok"])
                _smoke.run()
                smoke["ep_layer_ok"] = True
                report["ok"] = report["ok"] and smoke["invoke_rtt_ok"]
            except Exception as e:  # noqa: BLE001 - the report carries the failure
                smoke["error"] = f"{type(e).__name__}: {e}"
                report["ok"] = False
        report["smoke"] = smoke
    if args.json:
        print(json.dumps(report, indent=2, default=str))
    else:
        ext = report["extension"]
        print(f"kiwi_b200 {report['version']}: extension {'loaded' if ext['loaded'] else 'NOT loaded'}"
              + (f" ({ext.get('file')})" if ext["loaded"] else f": {ext.get('error')}"))
        e = report["env"]
        print(f"  torch {e.get('torch')}, CUDA runtime {e.get('cuda_runtime')}, NCCL {e.get('nccl')}, "
              f"driver {e.get('driver')}, commit {(e.get('repo') or {}).get('commit')}")
        if not report["gpus"]:
            print("  no CUDA device visible")
        for g in report["gpus"]:
            print(f"  GPU {g['index']}: {g['name']} (sm {g['capability']}, {g['sms']} SMs, {g['memory_gib']} GiB), "
                  f"P2P peers {g['p2p_peers']}, NVLS multicast {g['multicast']}")
        if "warning" in report:
            print("  warning: " + report["warning"])
        if "smoke" in report:
            print("  smoke: " + json.dumps(report["smoke"]))
        print("ok" if report["ok"] else "FAILED")
    return 0 if report["ok"] else 1


if __name__ == "__main__":
    sys.exit(main())
