"""Device collectives on one GPU: multi-round count all-to-all and barrier
(world 1), the reusable grid barrier under a cooperative launch, and a bounded
wait that runs out (a cell nothing writes) and reports kTimeout without
disturbing the context.  Reference test category: the collective-primitive and
timeout tests of apps/ep/tests (AMDResearch/kiwi)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

TIMEOUT = 2


@pytest.fixture(scope="module")
def coll():
    from kiwi_b200.parallel.collectives import DeviceCollectives
    from kiwi_b200.utils import dist as kdist

    kdist.init()
    return DeviceCollectives()


def test_all2all_rounds_world1(coll):
    send = torch.tensor([7], dtype=torch.int32, device="cuda")
    out = coll.all2all(send, rounds=50)
    torch.cuda.synchronize()
    coll.check()
    assert out[:, 0].tolist() == [7 + r for r in range(50)]
    assert int(coll.epoch.item()) == 50
    coll.barrier(rounds=10)
    torch.cuda.synchronize()
    coll.check()
    assert int(coll.epoch.item()) == 60


@pytest.mark.parametrize("blocks", [1, 37, 148])
def test_grid_barrier_rounds(blocks):
    from kiwi_b200.parallel.collectives import grid_barrier_test

    sms = torch.cuda.get_device_properties(0).multi_processor_count
    blocks = min(blocks, sms)
    r = grid_barrier_test(blocks, 200)
    assert r["status"] == 0, r
    assert r["word"] == 400 << 32, r  # 2 syncs per round, count back at zero


def test_bounded_wait_reports_timeout(coll):
    status = torch.zeros(2, dtype=torch.int32, device="cuda")
    waited = torch.zeros(1, dtype=torch.int64, device="cuda")
    coll.heap.native.coll_wait_only(coll.offset, 0x7ffffff0, 0, status, 50_000_000, waited)
    torch.cuda.synchronize()
    assert int(status[0].item()) != 0
    assert 40e6 < int(waited.item()) < 2e9
    # the context is still usable afterwards
    send = torch.tensor([1], dtype=torch.int32, device="cuda")
    coll.all2all(send)
    torch.cuda.synchronize()
    coll.check()
