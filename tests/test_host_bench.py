"""Host-only ring benchmark (two CPU threads ping-ponging over 4096 x 64 B rings), small sizes: checks order and checksum."""
import numpy as np

import kiwi_b200


def test_pingpong_small():
    C = kiwi_b200.native()
    r = C.bench.host_ring_pingpong(20000, 1000, 4096, 8, 0, -1, -1)
    assert r["ok"]
    lat = r["latencies_ns"]
    assert len(lat) == 20000 and np.all(lat > 0)


def test_stream_small_and_large_payload():
    C = kiwi_b200.native()
    assert C.bench.host_ring_stream(50000, 4096, 8, 3, -1, -1)["ok"]
    assert C.bench.host_ring_stream(2000, 256, 4096, 3, -1, -1)["ok"]


def test_xorshift_reference_values():
    C = kiwi_b200.native()
    # Marsaglia xorshift64 (13, 7, 17) from state 1.
    s = 1
    s ^= (s << 13) & (2**64 - 1)
    s ^= s >> 7
    s ^= (s << 17) & (2**64 - 1)
    assert C.bench.xorshift64(1) == s


def test_queue_baselines_all_designs_deliver_in_order():
    """Host-only queue baselines through one adapter contract (reference:
    benchmarks/queue_baselines): every design delivers in order with the
    right checksum, and reports latency and throughput."""
    from kiwi_b200._native import load

    rs = load().bench.queue_baselines(iters=2000, warmup=200, messages=20000, payload_bytes=8, capacity=64,
                                      idle_polls=100000, loaded=True)
    names = [r["name"] for r in rs]
    assert names == ["kiwi_ring", "head_tail", "seq_slot", "raw_word"]
    for r in rs:
        assert r["ok"], r
        assert r["p50_ns"] > 0 and r["p99_ns"] >= r["p50_ns"] and r["msgs_per_s"] > 0, r
        # idle poll and loaded ping-pong (reference modes idle-poll and loaded-latency)
        assert 0 < r["idle_poll_ns"] < 1e5, r
        assert r["loaded_p50_ns"] > 0 and r["loaded_p99_ns"] >= r["loaded_p50_ns"], r
        assert r["loaded_bg_msgs_per_s"] > 0, r
    plain = load().bench.queue_baselines(iters=200, warmup=20, messages=2000, capacity=64)
    assert "idle_poll_ns" not in plain[0] and "loaded_p50_ns" not in plain[0]
