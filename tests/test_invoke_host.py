"""kiwi::invoke on the host: registry, serialisation, dispatch, progress
threads.  Messages are enqueued by a CPU stand-in for the device
(reference: tests/invoke/test_invoke_basic.hip.cpp of AMDResearch/kiwi)."""
import struct
import threading
import time

import pytest

import kiwi_b200
from kiwi_b200 import invoke


def test_typed_callback_dispatch():
    ctx = invoke.Context(num_endpoints=2, capacity=64, host_only=True)
    got = []
    cb = ctx.register_callback(lambda a, b, c: got.append((a, b, c)), "<Qif")
    assert cb == 0
    ctx.emulate_invoke(1, cb, struct.pack("<Qif", 7, -3, 1.5))
    ctx.emulate_invoke(1, cb, struct.pack("<Qif", 8, 4, 2.5))
    assert ctx.progress(0) == 0
    assert ctx.progress(1) == 2
    assert got == [(7, -3, 1.5), (8, 4, 2.5)]


def test_raw_callback_any_size_and_order():
    ctx = invoke.Context(1, 256, host_only=True)
    seen = []
    cb = ctx.register_callback(lambda p: seen.append(p))
    msgs = [bytes([i % 256]) * i for i in range(0, 300, 7)]
    for m in msgs:
        ctx.emulate_invoke(0, cb, m)
    assert ctx.progress(0, max_callbacks=3) == 3
    ctx.progress(0)
    assert seen == msgs


def test_size_mismatch_raises():
    ctx = invoke.Context(1, 16, host_only=True)
    cb = ctx.register_callback(lambda a: None, "<Q")
    ctx.emulate_invoke(0, cb, b"1234")
    with pytest.raises(Exception, match="expects 8"):
        ctx.progress(0)


def test_unregistered_id_raises():
    ctx = invoke.Context(1, 16, host_only=True)
    ctx.emulate_invoke(0, 5, b"")
    with pytest.raises(Exception, match="unregistered"):
        ctx.progress(0)


def test_registry_limit_256():
    ctx = invoke.Context(1, 16, host_only=True)
    for i in range(invoke.MAX_CALLBACKS):
        assert ctx.register_callback(lambda p: None) == i
    with pytest.raises(Exception, match="full"):
        ctx.register_callback(lambda p: None)


def test_register_rejects_args_the_ring_cannot_hold():
    ctx = invoke.Context(1, 1, host_only=True)
    ctx.register_callback(lambda *a: None, "<3Q")  # 24 B: one line
    with pytest.raises(Exception, match="capacity"):
        ctx.register_callback(lambda *a: None, "<4Q")  # 32 B: two lines


def test_callback_exception_propagates():
    ctx = invoke.Context(1, 16, host_only=True)

    def boom(p):
        raise ValueError("boom")

    cb = ctx.register_callback(boom)
    ctx.emulate_invoke(0, cb, b"x")
    with pytest.raises(ValueError, match="boom"):
        ctx.progress(0)


def test_progress_threads_run_callbacks():
    ctx = invoke.Context(num_endpoints=4, capacity=64, host_only=True)
    lock = threading.Lock()
    seen = []

    def f(ep, i):
        with lock:
            seen.append((ep, i))

    cb = ctx.register_callback(f, "<II")
    ctx.start(num_threads=2)
    for i in range(50):
        for ep in range(4):
            while True:
                try:
                    ctx.emulate_invoke(ep, cb, struct.pack("<II", ep, i))
                    break
                except Exception:
                    time.sleep(0.001)
    deadline = time.time() + 10
    while len(seen) < 200 and time.time() < deadline:
        time.sleep(0.01)
    ctx.stop()
    assert len(seen) == 200
    for ep in range(4):
        assert [i for e, i in seen if e == ep] == list(range(50))


def test_progress_thread_error_surfaces():
    ctx = invoke.Context(1, 16, host_only=True)
    cb = ctx.register_callback(lambda p: 1 / 0)
    ctx.start(1)
    ctx.emulate_invoke(0, cb, b"")
    time.sleep(0.2)
    with pytest.raises(ZeroDivisionError):
        ctx.stop()


def test_mpsc_context_host_only():
    ctx = invoke.Context(1, 32, mpsc=True, host_only=True)
    got = []
    cb = ctx.register_callback(lambda v: got.append(v), "<d")
    ctx.emulate_invoke(0, cb, struct.pack("<d", 3.25))
    assert ctx.progress(0) == 1 and got == [3.25]


def test_progress_stats_and_affinity_log(capfd, monkeypatch):
    """Proxy counters (callbacks, sweeps, empty polls) and the
    KIWI_PROXY_AFFINITY_DEBUG log of each thread's CPUs and endpoints."""
    monkeypatch.setenv("KIWI_PROXY_AFFINITY_DEBUG", "1")
    ctx = invoke.Context(num_endpoints=3, capacity=64, host_only=True)
    got = []
    cb = ctx.register_callback(lambda i: got.append(i), "<I")
    cpus = kiwi_b200.native().topology.current_thread_cpus()
    ctx.start(num_threads=2, cpus=cpus[:1])
    for i in range(10):
        ctx.emulate_invoke(i % 3, cb, struct.pack("<I", i))
    deadline = time.time() + 10
    while len(got) < 10 and time.time() < deadline:
        time.sleep(0.01)
    st = ctx.stats
    assert st["threads"] == 2
    ctx.stop()
    st = ctx.stats
    assert sorted(got) == list(range(10))
    assert st["callbacks"] == 10 and st["threads"] == 0
    assert st["sweeps"] > 0 and st["empty_polls"] > 0
    err = capfd.readouterr().err
    lines = [ln for ln in err.splitlines() if ln.startswith("[kiwi] progress thread")]
    assert len(lines) == 2, err
    assert f"requested cpus {cpus[0]}, pinned 1, running on {cpus[0]}" in lines[0]
    assert "endpoints 0,2" in "".join(lines) and "endpoints 1" in "".join(lines)


def test_native_print_formats_packed_arguments():
    """Native print callback (reference: examples/common/kiwi_print_ext.hip.cpp):
    printf-style conversions over the packed argument image."""
    fmt = kiwi_b200.native().print_format.format
    pay = struct.pack("<ifQ", -3, 1.5, 0xC0FFEE03)
    assert fmt("step=%d value=%.2f tag=0x%llx", "<ifQ", pay) == "step=-3 value=1.50 tag=0xc0ffee03"
    assert fmt("%5u|%-4x|%c|%e", "IBbd", struct.pack("<IBbd", 7, 255, 65, 0.25)) == "    7|ff  |A|2.500000e-01"
    assert fmt("100%% of %hd and %lld", "hq", struct.pack("<hq", -2, 1 << 40)) == "100% of -2 and 1099511627776"
    assert fmt("unsigned %u", "Q", struct.pack("<Q", (1 << 64) - 1)) == "unsigned 18446744073709551615"
    assert fmt("no args %%", "", b"") == "no args %"
    for bad_fmt, codes in [("%s", "i"), ("%d", "f"), ("%f", "i"), ("%d %d", "i"), ("%d", "ii"), ("%*d", "i"),
                           ("%n", "i"), ("%d", "z"), ("tail %", "")]:
        with pytest.raises(Exception):
            fmt(bad_fmt, codes, b"\0" * 8)
    with pytest.raises(Exception):
        fmt("%d", "i", b"\0" * 3)  # wrong payload size


def test_native_print_callback_prints_each_invoke(capfd):
    ctx = invoke.Context(num_endpoints=1, capacity=64, host_only=True)
    cb = ctx.register_native_print("[kernel] step=%d value=%.2f tag=0x%llx", "<ifQ")
    for i in range(3):
        ctx.emulate_invoke(0, cb, struct.pack("<ifQ", i, i * 0.5, 0xC0FFEE00 + i))
    assert ctx.progress(0) == 3
    out = capfd.readouterr().out.splitlines()
    assert out[-3:] == ["[kernel] step=0 value=0.00 tag=0xc0ffee00", "[kernel] step=1 value=0.50 tag=0xc0ffee01",
                        "[kernel] step=2 value=1.00 tag=0xc0ffee02"]
    with pytest.raises(Exception):
        ctx.register_native_print("%s", "<i")


def test_load_cuda_builds_and_caches_a_kiwi_kernel_library(tmp_path):
    """kiwi_b200.utils.build.load_cuda: nvcc-only build of a source that uses
    the kiwi headers, loaded with ctypes (no GPU needed to build or call a host
    function); an unchanged source is not rebuilt."""
    import ctypes

    from kiwi_b200.utils.build import load_cuda

    src = r"""
#include <cstdint>
#include <kiwi/queue/wire.hpp>
__global__ void never_launched(uint32_t* out) { out[0] = kiwi::queue::wire_tag(threadIdx.x); }
extern "C" uint32_t kiwi_jit_tag(uint64_t n) { return kiwi::queue::wire_tag(n); }
"""
    lib = load_cuda("kiwi_jit_test", src, build_directory=str(tmp_path))
    lib.kiwi_jit_tag.argtypes = [ctypes.c_uint64]
    lib.kiwi_jit_tag.restype = ctypes.c_uint32
    assert lib.kiwi_jit_tag(0) == 1 and lib.kiwi_jit_tag(65535) == 1 and lib.kiwi_jit_tag(65534) == 65535
    so = tmp_path / "libkiwi_jit_test.so"
    mtime = so.stat().st_mtime_ns
    load_cuda("kiwi_jit_test", src, build_directory=str(tmp_path))
    assert so.stat().st_mtime_ns == mtime  # cached
    with pytest.raises(RuntimeError, match="nvcc failed"):
        load_cuda("kiwi_jit_bad", "this is not C++", build_directory=str(tmp_path / "bad"))


def test_progress_threads_poll_only_the_active_prefix():
    """Endpoints past the active prefix are not polled; growing the prefix
    reaches them; shrinking delivers what was already queued; stop() drains
    everything (the reference's active-queue state)."""
    import time

    ctx = invoke.Context(8, 16, host_only=True)
    got = []
    cb = ctx.register_callback(lambda p: got.append(p[0]))

    def wait_for(n):
        deadline = time.monotonic() + 10
        while len(got) < n and time.monotonic() < deadline:
            time.sleep(1e-3)

    ctx.set_active_endpoints(2)
    assert ctx.active_endpoints == 2
    ctx.start(num_threads=3, cpus=[])
    try:
        ctx.emulate_invoke(1, cb, b"\x01")
        ctx.emulate_invoke(5, cb, b"\x05")  # outside the prefix
        wait_for(1)
        time.sleep(0.05)
        assert got == [1]
        ctx.set_active_endpoints(0, wait_s=10)  # all endpoints
        wait_for(2)
        assert got == [1, 5]
        for ep in (3, 6, 7):
            ctx.emulate_invoke(ep, cb, bytes([ep]))
        ctx.set_active_endpoints(1, wait_s=10)  # shrink: the three queued messages arrive first
        assert sorted(got) == [1, 3, 5, 6, 7]
        ctx.emulate_invoke(4, cb, b"\x04")
        time.sleep(0.05)
        assert len(got) == 5
    finally:
        ctx.stop()
    assert sorted(got) == [1, 3, 4, 5, 6, 7]  # the final drain covers every endpoint


def test_a_kernel_can_publish_its_active_endpoints():
    """The active-prefix callback (what a kernel invokes with the number of
    endpoints it uses) sets the prefix the progress threads poll."""
    ctx = invoke.Context(4, 16, host_only=True)
    cb = ctx.register_active_endpoints_callback()
    ctx.emulate_invoke(0, cb, struct.pack("<I", 2))
    assert ctx.progress(0) == 1
    assert ctx.active_endpoints == 2
    ctx.emulate_invoke(1, cb, struct.pack("<I", 0))
    assert ctx.progress(1) == 1 and ctx.active_endpoints == 0
