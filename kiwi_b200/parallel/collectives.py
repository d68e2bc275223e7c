"""kiwi_b200.parallel.collectives: device-side count all-to-all and barrier over
NVLink (``include/kiwi/p2p/collectives.cuh``).

``DeviceCollectives(group)`` is collective.  It owns (or borrows, with
``heap`` and ``offset``) 2 x world 8-byte ingress cells in a symmetric heap and
a device epoch counter; every rank must issue the same sequence of
``all2all`` / ``barrier`` calls.  Each call is one single-block kernel on the
current stream (CUDA-graph capturable: the epoch lives on the device), with
bounded waits whose timeouts land in ``status`` (``check()`` raises).

Reference parity: the count all2all and cross-rank barrier of
apps/ep/all2all.hip.hpp:26-161 and apps/ep/barrier.hpp:23-54 (AMDResearch/kiwi).
"""
import torch

from .._native import load as _load
from ..utils import dist as kdist
from .p2p import SymmetricHeap

_C = _load()


class DeviceCollectives:
    """Device-side count all-to-all and cross-rank barrier over NVLink
    (``include/kiwi/p2p/collectives.cuh``): one u32 per (source, destination)
    pair per round, epoch-tagged ingress cells in a symmetric heap (its own
    2 MB heap unless `heap` and a 64-byte aligned `offset` are given), every wait
    bounded by `timeout_s`.  Collective constructor."""
    def __init__(self, group=None, heap=None, offset=0, timeout_s=5.0):
        self.group = group
        self.rank = kdist.rank(group)
        self.world = kdist.world_size(group)
        need = _C.p2p.coll_ingress_bytes(self.world)
        if heap is None:
            heap, offset = SymmetricHeap(max(need, 1 << 21), group), 0
        if offset % 64 or offset + need > heap.size:
            raise ValueError("ingress must be 64-byte aligned and inside the heap")
        self.heap = heap
        self.offset = int(offset)
        self.timeout_ns = int(timeout_s * 1e9)
        dev = torch.device("cuda", torch.cuda.current_device())
        heap.tensor(self.offset, [need // 4], torch.int32).zero_()
        self.epoch = torch.zeros(1, dtype=torch.int32, device=dev)
        self.status = torch.zeros(2, dtype=torch.int32, device=dev)
        torch.cuda.synchronize()
        kdist.barrier(group)

    def all2all(self, send, out=None, rounds=1, lat=None):
        """send: int32 [world] on this GPU (send[d] goes to rank d).  Returns
        recv int32 [rounds, world] (round r carries send + r)."""
        if out is None:
            out = torch.empty(rounds, self.world, dtype=torch.int32, device=send.device)
        self.heap.native.all2all_rounds(self.offset, send, out, self.epoch, self.status, self.timeout_ns, rounds, lat)
        return out

    def barrier(self, rounds=1, lat=None):
        self.heap.native.all2all_rounds(self.offset, None, None, self.epoch, self.status, self.timeout_ns, rounds, lat)

    def check(self):
        code, info = (int(v) for v in self.status.tolist())
        if code:
            raise RuntimeError(f"kiwi device collective failed: status={code} (late rank {info})")


def grid_barrier_test(blocks, rounds, timeout_s=2.0):
    """Cooperative-launch self test of the reusable grid barrier."""
    return _C.p2p.grid_barrier_test(int(blocks), int(rounds), int(timeout_s * 1e9))


__all__ = ["DeviceCollectives", "grid_barrier_test"]
