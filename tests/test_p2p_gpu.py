"""kiwi::p2p on one B200: symmetric heap mapping, the control plane (device
posts copy-engine puts and host signals that proxy threads execute), gets."""
import pytest
import torch

import kiwi_b200
from kiwi_b200.parallel.p2p import SymmetricHeap

pytestmark = pytest.mark.gpu


def test_heap_local_view_roundtrip():
    heap = SymmetricHeap(1 << 21)
    assert heap.size >= 1 << 21
    t = heap.tensor(4096, [1024], torch.float32)
    t.copy_(torch.arange(1024, device="cuda", dtype=torch.float32))
    assert heap.local_ptr == heap.peer_ptr(0)
    assert torch.equal(heap.tensor(4096, [1024], torch.float32).cpu(), torch.arange(1024, dtype=torch.float32))
    with pytest.raises(Exception):
        heap.tensor(heap.size - 8, [16], torch.float32)


@pytest.mark.parametrize("bytes_,n", [(64, 4), (1 << 20, 8)])
def test_control_plane_copy_engine_puts(bytes_, n):
    C = kiwi_b200.native()
    heap = SymmetricHeap(32 << 20)
    ctx = C.p2p.Context(heap.native, 1, 256)
    src_off, dst_off, flag_off, counter_off = 1 << 20, 4 << 20, 0, 256
    src = heap.tensor(src_off, [bytes_], torch.uint8)
    src.copy_(torch.randint(0, 256, (bytes_,), device="cuda", dtype=torch.uint8))
    heap.tensor(0, [512], torch.uint8).zero_()
    status = torch.zeros(2, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    ctx.spawn_proxy_threads(1)
    ctx.ce_put_selftest(0, src_off, dst_off, bytes_, n, flag_off, counter_off, status, 5_000_000_000)
    torch.cuda.synchronize()
    ctx.join_proxy_threads()
    assert int(status[0].item()) == 0, status
    assert ctx.copies_issued == n
    for i in range(n):
        assert torch.equal(heap.tensor(dst_off + i * bytes_, [bytes_], torch.uint8), src)
    assert int(heap.tensor(flag_off, [1], torch.int64).item()) == n
    assert int(heap.tensor(flag_off + 8, [1], torch.int64).item()) == 0xABCD


def test_proxy_threads_serve_the_active_queue_prefix():
    """Four control queues, proxies restricted to queue 0 (the one the
    self-test kernel's single block posts on): every put is still served."""
    C = kiwi_b200.native()
    heap = SymmetricHeap(8 << 20)
    ctx = C.p2p.Context(heap.native, 4, 256)
    gen = ctx.set_active_queues(1)
    src_off, dst_off = 1 << 20, 2 << 20
    heap.tensor(src_off, [4096], torch.uint8).fill_(7)
    heap.tensor(0, [512], torch.uint8).zero_()
    status = torch.zeros(2, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    ctx.spawn_proxy_threads(2)
    ctx.ce_put_selftest(0, src_off, dst_off, 4096, 3, 0, 256, status, 5_000_000_000)
    torch.cuda.synchronize()
    assert ctx.active_applied(gen)
    ctx.join_proxy_threads()
    assert int(status[0].item()) == 0, status
    assert ctx.copies_issued == 3
    assert bool((heap.tensor(dst_off, [3 * 4096], torch.uint8) == 7).all())


def test_get_from_own_heap():
    heap = SymmetricHeap(4 << 20)
    n = 1 << 20
    src = heap.tensor(0, [n], torch.uint8)
    src.copy_(torch.randint(0, 256, (n,), device="cuda", dtype=torch.uint8))
    lat = torch.zeros(3, dtype=torch.int64, device="cuda")
    heap.native.get(0, n, 3, 0, 2 << 20, lat, 64)
    torch.cuda.synchronize()
    assert torch.equal(heap.tensor(2 << 20, [n], torch.uint8), src)


def test_completion_counter_host_signals_kernel():
    """A kernel polls a completion counter (bounded) while a host thread bumps
    it; every value is seen, in order."""
    import threading
    import time

    C = kiwi_b200.native()
    c = C.p2p.CompletionCounter()
    steps = 200
    seen = torch.zeros(steps, dtype=torch.int64, device="cuda")
    status = torch.zeros(2, dtype=torch.int32, device="cuda")
    c.wait_kernel(steps, seen, status, 5_000_000_000)

    def bump():
        for _ in range(steps):
            c.signal()
            time.sleep(20e-6)

    t = threading.Thread(target=bump)
    t.start()
    t.join()
    torch.cuda.synchronize()
    assert int(status[0].item()) == 0, status
    s = seen.cpu()
    assert bool((s[1:] >= s[:-1]).all())
    assert c.get() == steps


def test_completion_counter_wait_times_out():
    """Nobody signals: the kernel's wait returns kTimeout after its deadline
    and the context stays usable."""
    C = kiwi_b200.native()
    c = C.p2p.CompletionCounter()
    seen = torch.zeros(1, dtype=torch.int64, device="cuda")
    status = torch.zeros(2, dtype=torch.int32, device="cuda")
    c.wait_kernel(1, seen, status, 50_000_000)
    torch.cuda.synchronize()
    assert int(status[0].item()) != 0
    assert torch.ones(1, device="cuda").item() == 1.0


def test_checked_mode_records_and_skips_out_of_range_accesses():
    """Checked mode: every rejected range lies past the checked limit but
    inside the mapped heap, so even a broken check could not leave the
    mapping.  Rejected puts, gets and signals leave memory untouched and the
    first violation is reported; valid ones run unchanged."""
    heap = SymmetricHeap(4 << 20)
    limit = 1 << 20
    heap.enable_checks(limit)
    assert heap.native.check_limit == limit
    n = 4096
    src = heap.tensor(0, [n], torch.uint8)
    src.copy_(torch.randint(1, 256, (n,), device="cuda", dtype=torch.uint8))
    flag = heap.tensor(512 << 10, [1], torch.int64)
    flag.zero_()
    # valid: put to 64 KiB, get back to [n, 2n), signal the flag
    heap.native.checked_ops(0, 64 << 10, n, 512 << 10)
    torch.cuda.synchronize()
    assert heap.check_error() is None
    assert torch.equal(heap.tensor(64 << 10, [n], torch.uint8), src)
    assert torch.equal(heap.tensor(n, [n], torch.uint8), src)
    assert flag.item() == 1
    # put / get crossing the limit: skipped, recorded as a put at that offset
    edge = limit - 1024
    beyond = heap.tensor(edge, [n], torch.uint8)
    beyond.zero_()
    heap.tensor(n, [n], torch.uint8).zero_()
    heap.native.checked_ops(0, edge, n, 512 << 10)
    torch.cuda.synchronize()
    assert heap.check_error() == {"site": "put", "rank": 0, "offset": edge}
    assert int(beyond.count_nonzero()) == 0
    assert int(heap.tensor(n, [n], torch.uint8).count_nonzero()) == 0  # the get was skipped too
    assert flag.item() == 2  # the valid signal still ran
    # signal past the limit: skipped and recorded
    heap.clear_check_error()
    far = heap.tensor(2 << 20, [1], torch.int64)
    far.zero_()
    heap.native.checked_ops(0, 64 << 10, 0, 2 << 20)
    torch.cuda.synchronize()
    assert heap.check_error() == {"site": "signal", "rank": 0, "offset": 2 << 20}
    assert far.item() == 0
    heap.disable_checks()
    assert heap.check_error() is None
