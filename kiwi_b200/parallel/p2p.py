"""kiwi_b200.parallel.p2p: NVLink symmetric heap and device-initiated P2P.

``SymmetricHeap(nbytes, group)`` is collective: every rank allocates ``nbytes``
of device memory with ``cuMemCreate``, the ranks exchange POSIX file
descriptors over abstract Unix sockets and map each other's memory, so a kernel
on rank r can store straight into rank q's heap (``include/kiwi/p2p/device.cuh``:
put / get / signal / wait).  With ``multicast=True`` an NVLS multicast object is
bound over all heaps (``multimem.st`` broadcast, ``multimem.ld_reduce``).

Reference parity: ``register_symmetric`` and ``ghandle_t::post_put`` /
``post_p`` (apps/p2p/context.hip.{hpp,cpp} of AMDResearch/kiwi), which go
through CPU proxy threads and RDMA; here the data path is the kernel itself.
"""
import torch

from .._native import load as _load
from ..utils import dist as kdist

_C = _load()


class SymmetricHeap:
    """`nbytes` of device memory on every rank of `group`, mapped into every
    rank's address space over NVLink (collective constructor).  ``native.view()``
    is the by-value ``HeapView`` kernels take; ``tensor(offset, shape, dtype)`` a
    torch view of this rank's part; ``enable_checks(limit)`` the checked mode of
    the device put / get / signal API."""
    def __init__(self, nbytes, group=None, multicast=False, timeout_s=60.0):
        self.group = group
        self.rank = kdist.rank(group)
        self.world = kdist.world_size(group)
        device = torch.cuda.current_device()
        job = kdist.job_id(group)
        if multicast and not _C.p2p.multicast_supported(device):
            raise RuntimeError("NVLS multicast is not supported on this device")

        def _barrier():
            kdist.barrier(group)

        self._h = _C.p2p.SymmetricHeap(device, int(nbytes), self.rank, self.world, job, bool(multicast), _barrier)
        kdist.barrier(group)

    @property
    def native(self):
        return self._h

    @property
    def size(self):
        return self._h.size

    @property
    def local_ptr(self):
        return self._h.local_ptr

    @property
    def mc_ptr(self):
        return self._h.mc_ptr

    def peer_ptr(self, rank):
        return self._h.peer_ptr(rank)

    def tensor(self, offset, shape, dtype):
        """A torch view of this rank's heap (local memory only)."""
        if isinstance(shape, int):
            shape = [shape]
        return self._h.tensor(int(offset), list(shape), dtype)

    # -- checked mode ------------------------------------------------------------
    def enable_checks(self, limit=None):
        """Validate every put / get / signal of the device API against
        [0, limit) of a valid rank's heap (default: the whole heap).  A bad
        access is skipped and the first one recorded (see :meth:`check_error`);
        nothing traps.  Applies to kernels launched with views taken after the
        call, i.e. every launch from here on."""
        dev = torch.device("cuda", torch.cuda.current_device())
        self._check = torch.zeros(4, dtype=torch.int32, device=dev)
        self._h.set_checks(self._check, int(limit or 0))

    def disable_checks(self):
        self._h.set_checks(None)
        self._check = None

    def check_error(self):
        """None, or {"site", "rank", "offset"} of the first rejected access
        (offset: low 32 bits).  Synchronises the current stream."""
        rec = getattr(self, "_check", None)
        if rec is None:
            return None
        code, site, rank, off = (int(v) for v in rec.cpu().tolist())
        if code == 0:
            return None
        return {"site": _C.p2p.CheckSite(site).name.lower(), "rank": rank, "offset": off & 0xFFFFFFFF}

    def clear_check_error(self):
        if getattr(self, "_check", None) is not None:
            self._check.zero_()

    def barrier(self, flag_offset, round_, status):
        """Device-side barrier over the heap: flag words at flag_offset + 8*rank."""
        self._h.barrier(int(flag_offset), int(round_), status, 2_000_000_000)


def exchange_fds(job, rank, world, fd, timeout_s=60.0):
    """Every rank passes one file descriptor and receives every rank's (in
    rank order), over abstract Unix sockets named after `job`."""
    return _C.p2p.exchange_fds(job, rank, world, fd, timeout_s)


__all__ = ["SymmetricHeap", "exchange_fds"]
