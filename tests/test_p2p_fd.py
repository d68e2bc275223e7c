"""FD exchange over abstract Unix sockets between processes (CPU only):
the bootstrap the symmetric heap uses, tested with memfd objects."""
import multiprocessing as mp
import os
import uuid

import pytest


def _worker(job, rank, world, q):
    import kiwi_b200

    C = kiwi_b200.native()
    fd = os.memfd_create(f"kiwi-test-{rank}")
    os.write(fd, f"rank{rank}".encode())
    try:
        fds = C.p2p.exchange_fds(job, rank, world, fd, 20.0)
        got = []
        for f in fds:
            # pread: descriptors passed with SCM_RIGHTS share one file offset
            # across processes, so seek + read would race with the peers.
            got.append(os.pread(f, 16, 0).decode())
            os.close(f)
        q.put((rank, got))
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e)))


@pytest.mark.parametrize("world", [2, 4])
def test_exchange_fds(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    job = uuid.uuid4().hex[:12]
    ps = [ctx.Process(target=_worker, args=(job, r, world, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in ps:
        p.join(timeout=60)
    for r in range(world):
        assert res[r] == [f"rank{i}" for i in range(world)], res[r]


def _lonely(job, q):
    import kiwi_b200

    C = kiwi_b200.native()
    fd = os.memfd_create("kiwi-lonely")
    try:
        C.p2p.exchange_fds(job, 0, 2, fd, 1.0)
        q.put("no error")
    except Exception as e:
        q.put(str(e))


def test_missing_peer_times_out():
    """A rank that never joins makes the exchange fail after its timeout (no hang)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely, args=(uuid.uuid4().hex[:12], q))
    p.start()
    msg = q.get(timeout=60)
    p.join(timeout=30)
    assert "timed out" in msg


def test_completion_counter_host_only():
    """Completion counter (reference: apps/p2p/comp_counter.hip.hpp): host
    threads signal with release fetch_add, the value is monotonic."""
    import threading

    from kiwi_b200._native import load

    c = load().p2p.CompletionCounter(host_only=True)
    assert c.get() == 0
    ths = [threading.Thread(target=lambda: [c.signal() for _ in range(10000)]) for _ in range(4)]
    for t in ths:
        t.start()
    for t in ths:
        t.join()
    assert c.get() == 40000
    c.set(7)
    assert c.signal(3) == 10


def test_checked_mode_range_rule():
    """The device API's checked mode rejects an access unless the rank exists
    and [off, off + bytes) stays inside the checked limit (overflow included)."""
    from kiwi_b200._native import load

    ok = load().p2p.heap_range_ok
    lim = 1 << 20
    assert ok(2, lim, 0, 0, lim)
    assert ok(2, lim, 1, lim - 96, 96)
    assert ok(2, lim, 1, lim, 0)
    assert not ok(2, lim, 1, lim - 96, 97)
    assert not ok(2, lim, 2, 0, 8)
    assert not ok(2, lim, -1, 0, 8)
    assert not ok(2, lim, 0, lim + 1, 0)
    assert not ok(2, lim, 0, 8, (1 << 64) - 4)  # off + bytes would wrap
    sites = load().p2p.CheckSite
    assert [sites.PUT.value, sites.GET.value, sites.SIGNAL.value] == [1, 2, 3]
