"""kiwi::queue on a B200: every push path and size through both device-to-host
queues, relaunch with saved handles, the host-to-device queues, bounded waits,
and the register-resident (no local memory) contract.

Mirrors the reference's GPU queue tests (tests/queue/test_chunk_queue.hip.cpp,
test_push_lane_masked, test_host_to_device_concurrent,
test_queue_mpmc_h2d_concurrent, check_push_isa.cmake of AMDResearch/kiwi).
"""
import pytest

import kiwi_b200

pytestmark = pytest.mark.gpu


def _C():
    return kiwi_b200.native()


def _ok(r):
    assert r["mismatches"] == 0, r
    assert r["order_errors"] == 0, r
    assert r["device_error"] == 0, r
    assert r["first_error"] == "", r


@pytest.mark.parametrize("cap", [1, 4, 64, 4096])
def test_spsc_global_small_sizes(cap):
    sizes = [s for s in [0, 1, 7, 8, 9, 24, 25, 56, 100] if (s + 8 + 31) // 32 <= cap]
    r = _C().bench.d2h_push_test("global", False, cap, 1, 300, sizes, 1, 11)
    _ok(r)
    assert r["popped"] == 300


def test_spsc_global_all_sizes_to_4k():
    sizes = list(range(0, 520, 13)) + [1000, 2047, 2048, 4095, 4096]
    r = _C().bench.d2h_push_test("global", False, 256, 1, 2 * len(sizes), sizes, 2, 12)
    _ok(r)


def test_spsc_lanes_and_relaunch():
    sizes = [0, 8, 24, 64, 128, 248, 256]
    r = _C().bench.d2h_push_test("lanes", False, 16, 1, 200, sizes, 3, 13)
    _ok(r)
    assert r["popped"] == 600


@pytest.mark.parametrize("size", [8, 20, 56, 200, 512])
def test_spsc_reg(size):
    r = _C().bench.d2h_push_test("reg", False, 32, 1, 100, [size], 1, 14)
    _ok(r)


@pytest.mark.parametrize("cap", [128, 1024])
def test_spsc_lane_masked(cap):
    r = _C().bench.d2h_push_test("lane_masked", False, cap, 1, 20, [8], 2, 15)
    _ok(r)
    assert r["popped"] > 0


@pytest.mark.parametrize("warps,cap", [(8, 16), (64, 64), (304, 8)])
def test_mpsc_many_warps(warps, cap):
    r = _C().bench.d2h_push_test("global", True, cap, warps, 20, [8, 24, 100], 1, 16)
    _ok(r)
    assert r["popped"] == warps * 20


def test_mpsc_lanes_and_lane_masked():
    _ok(_C().bench.d2h_push_test("lanes", True, 32, 16, 30, [16, 200], 1, 17))
    _ok(_C().bench.d2h_push_test("lane_masked", True, 256, 8, 5, [8], 1, 18))


@pytest.mark.parametrize("registers", [True, False])
def test_h2d_spsc(registers):
    sizes = [0, 8, 24, 56, 200, 248] if registers else [0, 8, 100, 1000, 4096]
    cap = 16 if registers else 256
    r = _C().bench.h2d_spsc_test(cap, 300, sizes, registers, 1, 21)
    _ok(r)
    assert r["popped"] == 300


def test_h2d_spsc_batched_notify():
    r = _C().bench.h2d_spsc_test(64, 500, [8, 56], True, 16, 22)
    _ok(r)


@pytest.mark.parametrize("slots,slot_lines,producers,warps", [(4, 1, 1, 1), (16, 2, 4, 8), (64, 8, 3, 32)])
def test_h2d_mpmc(slots, slot_lines, producers, warps):
    r = _C().bench.h2d_mpmc_test(slots, slot_lines, producers, 300, warps, 23)
    _ok(r)
    assert r["popped"] == producers * 300


def test_bounded_wait_times_out():
    # Nothing is ever pushed: the device pop must give up with kTimeout (1) and record it.
    assert _C().bench.h2d_timeout_test(20_000_000) == 1


def test_hot_path_kernels_use_no_local_memory():
    attrs = _C().bench.queue_kernel_attributes()
    for name, local, regs in attrs:
        assert local == 0, f"{name} uses {local} B of local memory"


def test_invoke_roundtrip_small():
    r = _C().bench.invoke_rtt(iters=2000, warmup=200, payload_bytes=8)
    assert r["ok"], r
    assert r["callbacks"] == 2200
    r = _C().bench.invoke_rtt(iters=500, warmup=50, payload_bytes=4096, capacity=512)
    assert r["ok"], r
    r = _C().bench.invoke_rtt(iters=500, warmup=50, payload_bytes=8, mpsc=True)
    assert r["ok"], r
    r = _C().bench.invoke_rtt(iters=2000, warmup=200, payload_bytes=8, poll_warps=4)
    assert r["ok"], r


def test_pcie_floor_small():
    r = _C().bench.pcie_floor(iters=2000, warmup=200)
    assert r["ok"], r


@pytest.mark.parametrize("mode", [0, 1, 3, 6, 7, 8])
def test_platform_rewritten_words_read_old_new_or_zero(mode):
    """The wire format's hardware assumption (reference category:
    tests/queue/test_hardware_assumptions.hip.cpp): while a kernel rewrites a
    line of mapped host memory back to back, a host 8-byte load returns, per
    4-byte word, the old value, the new value or zero (B200 hosts show
    transient zeros; never a mix of the two values).  Modes are listed in
    csrc/queue_gpu.cu."""
    r = _C().bench.atomicity_test(1_000_000, mode)
    assert r["final_ok"], r
    assert r["reads"] > 1000, r
    assert r["torn_nonzero"] == 0, r


def test_platform_host_rewrites_seen_by_gpu():
    """Host -> device direction: a GPU 16-byte load of a line the host keeps
    rewriting sees each word old, new or zero."""
    r = _C().bench.atomicity_h2d_test(1500)
    assert r["final_ok"], r
    assert r["reads"] > 1000, r
    assert r["torn_nonzero"] == 0, r


@pytest.mark.parametrize("fmt", [0, 1])
def test_ring_reader_never_accepts_stale_data(fmt):
    """A ring reader's view: the GPU writes round i once, the host waits for
    round i's tags and checks the data of every half that carries them."""
    r = _C().bench.atomicity_protocol_test(200_000, fmt)
    assert r["ok"], r
    assert r["accepted_bad"] == 0, r


def test_invoke_throughput_and_push_cost():
    C = _C()
    r = C.bench.invoke_throughput(endpoints=8, threads=2, msgs_per_endpoint=20000, payload_bytes=8)
    assert r["ok"], r
    assert r["messages"] == 8 * 20000
    c = C.bench.push_cost(20000, 8)
    assert c["ok"] and c["cycles_per_push"] > 0, c
