"""Environment provenance for benchmark and profiling runs.

    python -m kiwi_b200.utils.env [--output FILE]

Collects, read-only, what a measurement depends on: host and CPU, Python,
PyTorch / CUDA / NCCL versions, the NVIDIA driver and each visible GPU (name,
memory, SM count, PCI bus, NUMA node, current and maximum SM clocks, power
limit, active clock-event reasons), the repository commit, and the KIWI_*,
NCCL_* and CUDA_* variables.  Nothing here changes a setting.

Parity: the reference's provenance script for EP benchmark runs
(scripts/ep_bench/collect_env.sh of AMDResearch/kiwi), which records the
host, ROCm, MPI, Python, image and source details of a run.
"""
import datetime
import json
import os
import platform
import socket
import subprocess
import sys

_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
_ENV_PREFIXES = ("KIWI_", "NCCL_", "CUDA_", "TORCH_NCCL_")


def _git(*args):
    try:
        r = subprocess.run(["git", "-C", _ROOT, *args], capture_output=True, text=True, timeout=10)
        return r.stdout.strip() if r.returncode == 0 else None
    except (OSError, subprocess.SubprocessError):
        return None


def _cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or None


def _torch_info():
    try:
        import torch
    except ImportError:
        return {"torch": None}
    d = {"torch": torch.__version__, "cuda_runtime": torch.version.cuda, "cuda_available": torch.cuda.is_available()}
    try:
        v = torch.cuda.nccl.version()
        d["nccl"] = ".".join(str(x) for x in v) if isinstance(v, tuple) else str(v)
    except Exception:  # noqa: BLE001 - not built with NCCL, or no CUDA
        d["nccl"] = None
    return d


def _nvml_gpus():
    """Per-GPU read-only NVML queries; [] without a driver."""
    try:
        import pynvml as nv
    except ImportError:
        return None, []
    try:
        nv.nvmlInit()
    except Exception:  # noqa: BLE001 - no driver on this host
        return None, []
    gpus = []
    try:
        driver = nv.nvmlSystemGetDriverVersion()
        driver = driver.decode() if isinstance(driver, bytes) else driver
        for i in range(nv.nvmlDeviceGetCount()):
            h = nv.nvmlDeviceGetHandleByIndex(i)
            name = nv.nvmlDeviceGetName(h)
            g = {"index": i, "name": name.decode() if isinstance(name, bytes) else name}
            for key, fn in (("memory_total_mib", lambda: nv.nvmlDeviceGetMemoryInfo(h).total // (1 << 20)),
                            ("sm_clock_mhz", lambda: nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                            ("sm_clock_max_mhz", lambda: nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)),
                            ("power_limit_w", lambda: nv.nvmlDeviceGetEnforcedPowerLimit(h) / 1000.0),
                            ("clock_event_reasons", lambda: int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))),
                            ("pci_bus_id", lambda: _str(nv.nvmlDeviceGetPciInfo(h).busId))):
                try:
                    g[key] = fn()
                except Exception:  # noqa: BLE001 - a field this driver does not report
                    g[key] = None
            gpus.append(g)
    finally:
        try:
            nv.nvmlShutdown()
        except Exception:  # noqa: BLE001
            pass
    return driver, gpus


def _str(v):
    return v.decode() if isinstance(v, bytes) else v


def _torch_gpus():
    try:
        import torch
        if not torch.cuda.is_available():
            return []
        out = []
        for i in range(torch.cuda.device_count()):
            p = torch.cuda.get_device_properties(i)
            out.append({"index": i, "name": p.name, "sm_count": p.multi_processor_count,
                        "capability": f"{p.major}.{p.minor}", "memory_total_mib": p.total_memory // (1 << 20)})
        return out
    except Exception:  # noqa: BLE001
        return []


def _numa_nodes(gpus):
    try:
        from .._native import load
        topo = load().topology
    except Exception:  # noqa: BLE001 - extension not built
        return
    for g in gpus:
        try:
            g["numa_node"] = topo.gpu_numa_node(g["index"])
        except Exception:  # noqa: BLE001
            g["numa_node"] = None


def collect_env():
    """A JSON-serialisable dict of the run's environment (read-only)."""
    driver, nvml = _nvml_gpus()
    tgpus = _torch_gpus()
    by_index = {g["index"]: dict(g) for g in tgpus}
    for g in nvml:
        by_index.setdefault(g["index"], {}).update({k: v for k, v in g.items() if v is not None})
    gpus = [by_index[i] for i in sorted(by_index)]
    _numa_nodes(gpus)
    try:
        affinity = sorted(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        affinity = None
    return {
        "time_utc": datetime.datetime.now(datetime.timezone.utc).isoformat(timespec="seconds"),
        "host": socket.gethostname(),
        "platform": platform.platform(),
        "cpu": {"model": _cpu_model(), "count": os.cpu_count(), "affinity": affinity},
        "python": sys.version.split()[0],
        **_torch_info(),
        "driver": driver,
        "gpus": gpus,
        "repo": {"commit": _git("rev-parse", "HEAD"), "dirty": bool(_git("status", "--porcelain"))},
        "env": {k: v for k, v in sorted(os.environ.items()) if k.startswith(_ENV_PREFIXES)},
    }


def main(argv=None):
    """Command-line entry: prints (or writes) collect_env() as JSON."""
    import argparse

    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--output", default=None, help="write the JSON here instead of stdout")
    args = ap.parse_args(argv)
    text = json.dumps(collect_env(), indent=2, default=str)
    if args.output:
        with open(args.output, "w") as f:
            f.write(text + "\n")
    else:
        print(text)


if __name__ == "__main__":
    main()
