"""GPU-producer queue comparators (csrc/queue_baselines_gpu.cu): every queue
delivers every message once, in per-producer order, with its check word, in
each mode it supports; bad arguments are refused before any device work."""
import pytest

import kiwi_b200

C = kiwi_b200.native()


@pytest.mark.gpu
@pytest.mark.parametrize("queue", ["kiwi_spsc", "kiwi_mpsc", "fifo_trigger", "proxy_channel", "raw_store"])
def test_latency_mode_delivers_every_message(queue):
    r = C.bench.gpu_queue_baseline(queue, "latency", iters=2000, warmup=200, capacity=64)
    assert r["ok"], r
    assert r["messages"] == 2200 and len(r["lat_ns"]) == 2000
    assert 0 < float(r["lat_ns"].mean()) < 100_000


@pytest.mark.gpu
@pytest.mark.parametrize("queue,warps", [("kiwi_spsc", 1), ("kiwi_mpsc", 16), ("fifo_trigger", 16),
                                         ("proxy_channel", 16)])
def test_throughput_mode_keeps_per_producer_order(queue, warps):
    r = C.bench.gpu_queue_baseline(queue, "throughput", iters=3000, warps=warps, capacity=256)
    assert r["ok"], r
    assert r["messages"] == 3000 * warps and r["seconds"] > 0 and r["cycles_per_push"] > 0


@pytest.mark.gpu
@pytest.mark.parametrize("queue", ["kiwi_spsc", "fifo_trigger", "proxy_channel"])
def test_push_cost_mode_never_wraps(queue):
    r = C.bench.gpu_queue_baseline(queue, "push_cost", iters=2000, warps=1, capacity=4096)
    assert r["ok"], r
    assert r["cycles_per_push"] > 0


@pytest.mark.parametrize("kwargs", [
    dict(queue="mscclpp"),                                          # unknown queue
    dict(queue="kiwi_spsc", mode="stream"),                         # unknown mode
    dict(queue="kiwi_spsc", mode="throughput", warps=4),            # one producer warp only
    dict(queue="raw_store", mode="throughput"),                     # no capacity check: latency only
    dict(queue="fifo_trigger", capacity=1000),                      # not a power of two
    dict(queue="fifo_trigger", mode="push_cost", iters=100, warps=64, capacity=1024),  # would wrap
])
def test_bad_arguments_are_refused_before_device_work(kwargs):
    with pytest.raises(Exception):
        C.bench.gpu_queue_baseline(**kwargs)
