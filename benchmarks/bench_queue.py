"""Queue-level benchmarks on one B200 (reference: benchmarks/queue/*.hip.cpp and
benchmarks/invoke/bench_{throughput,overhead}.hip.cpp of AMDResearch/kiwi).

    python benchmarks/bench_queue.py

* host_ring: two CPU threads ping-pong 1,000,000 seeded 8-byte payloads through
  two 4096 x 64 B rings (the host-only ring benchmark), p50 / p99 round trip ns, order and
  checksum verified; plus a one-way streaming rate.
* queue_baselines: the same two-thread ping-pong and stream through four queue
  designs behind one adapter contract (kiwi ring, head/tail-counter ring,
  per-slot sequence ring, single-word floor), plus the cost of one poll of an
  empty queue and the ping-pong under a concurrent stream; reference:
  benchmarks/queue_baselines.
* gpu_queue_baseline: the device-producer comparators (this repository's SPSC
  and MPSC rings, an index-publishing trigger FIFO in the style of MSCCL++'s
  proxy FIFO, a lap-parity proxy channel in the style of NVSHMEM's, and the
  raw-store floor) in latency, throughput (W warps, one host consumer) and
  push-cost modes; reference: benchmarks/queue_baselines (GPU side).
* invoke_throughput: E producer warps x T progress threads, messages/s.
* push_cost: SM cycles one warp spends per push (payload 8 .. 256 B).
"""
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import numpy as np  # noqa: E402

import kiwi_b200  # noqa: E402


def emit(d):
    print("RESULT " + json.dumps(d), flush=True)


def main():
    C = kiwi_b200.native()
    cpus = C.topology.process_cpus()
    a, b = (cpus[1], cpus[2]) if len(cpus) > 2 else (-1, -1)
    r = C.bench.host_ring_pingpong(1_000_000, 10_000, 4096, 8, 0, a, b)
    lat = np.asarray(r["latencies_ns"])
    emit({"bench": "host_ring_pingpong", "ok": r["ok"], "messages": 1_000_000, "slots": 4096, "slot_bytes": 64,
          "p50_ns": float(np.percentile(lat, 50)), "p99_ns": float(np.percentile(lat, 99)), "cpus": [a, b]})
    s = C.bench.host_ring_stream(1_000_000, 4096, 8, 0, a, b)
    emit({"bench": "host_ring_stream", "ok": s["ok"], "Mmsg_per_s": 1e3 / s["total_ns"] * 1e6})
    # The loaded mode's background pair takes the two cores after the ping-pong's, when there are any.
    c_bg, d_bg = (cpus[3], cpus[4]) if len(cpus) > 4 else (-1, -1)
    for q in C.bench.queue_baselines(iters=200_000, warmup=20_000, messages=1_000_000, payload_bytes=8,
                                     capacity=4096, cpu_a=a, cpu_b=b, idle_polls=10_000_000, loaded=True,
                                     cpu_c=c_bg, cpu_d=d_bg):
        emit({"bench": "queue_baseline", "design": q["name"], "ok": q["ok"], "p50_ns": q["p50_ns"],
              "p99_ns": q["p99_ns"], "Mmsg_per_s": q["msgs_per_s"] / 1e6, "idle_poll_ns": q["idle_poll_ns"],
              "loaded_p50_ns": q["loaded_p50_ns"], "loaded_p99_ns": q["loaded_p99_ns"],
              "loaded_bg_Mmsg_per_s": q["loaded_bg_msgs_per_s"] / 1e6})
    if not C.cuda_device_available():
        return
    for q in ("kiwi_spsc", "kiwi_mpsc", "fifo_trigger", "proxy_channel", "raw_store"):
        r = C.bench.gpu_queue_baseline(q, "latency", iters=100_000, warmup=10_000, capacity=4096)
        lat = np.asarray(r["lat_ns"], dtype=np.float64)
        emit({"bench": "gpu_queue_baseline", "queue": q, "mode": "latency", "ok": r["ok"],
              "p50_us": float(np.percentile(lat, 50)) / 1e3, "p99_us": float(np.percentile(lat, 99)) / 1e3})
    for q in ("kiwi_spsc", "kiwi_mpsc", "fifo_trigger", "proxy_channel"):
        for w in ((1,) if q == "kiwi_spsc" else (1, 16, 64)):
            r = C.bench.gpu_queue_baseline(q, "throughput", iters=50_000, warps=w, capacity=4096)
            emit({"bench": "gpu_queue_baseline", "queue": q, "mode": "throughput", "warps": w, "ok": r["ok"],
                  "Mmsg_per_s": r["messages"] / max(r["seconds"], 1e-9) / 1e6,
                  "cycles_per_push": r["cycles_per_push"]})
        r = C.bench.gpu_queue_baseline(q, "push_cost", iters=20_000, warps=1, capacity=32768)
        emit({"bench": "gpu_queue_baseline", "queue": q, "mode": "push_cost", "ok": r["ok"],
              "cycles_per_push": r["cycles_per_push"]})
    for e, t in [(1, 1), (4, 1), (8, 2), (16, 4), (64, 4)]:
        r = C.bench.invoke_throughput(e, t, 20000, 8, 4096)
        emit({"bench": "invoke_throughput", "endpoints": e, "threads": t, "ok": r["ok"],
              "Mmsg_per_s": r["messages"] / max(r["device_ns"], 1) * 1e3})
    for nbytes in [8, 32, 64, 128, 256]:
        c = C.bench.push_cost(20000, nbytes)
        emit({"bench": "push_cost", "payload_bytes": nbytes, "ok": c["ok"], "cycles": c["cycles_per_push"]})


if __name__ == "__main__":
    main()
