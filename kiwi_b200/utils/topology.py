"""CPU / NUMA placement of a rank next to its GPU.

``bind_process_to_gpu(device)`` restricts the calling process to the CPUs of the
GPU's NUMA node (intersected with the CPUs the process may use), so that pinned
host buffers allocated afterwards (``cudaHostAlloc`` places pages on the
allocating thread's node) and the host threads that poll them sit on the
GPU-local socket.  Reference behaviour: the GPU-local affinity helpers of
include/kiwi/common/topology.hpp and src/common/topology.cpp in AMDResearch/kiwi.
"""
import os

from .._native import load as _load


def gpu_local_cpus(device):
    """CPUs local to CUDA device `device` that this process may run on; all the
    CPUs it may run on when the device's local CPUs are unknown (no GPU, no
    sysfs entry) or none of them is allowed."""
    local = set(_load().topology.gpu_local_cpus(int(device)))
    allowed = os.sched_getaffinity(0)
    return sorted(local & allowed)


def bind_process_to_gpu(device):
    """Restricts this process to `device`'s local CPUs and returns them.  When
    those are unknown or not allowed, :func:`gpu_local_cpus` returns every CPU
    the process may already use, so the affinity does not change."""
    cpus = gpu_local_cpus(device)
    if cpus:
        os.sched_setaffinity(0, cpus)
    return cpus


__all__ = ["gpu_local_cpus", "bind_process_to_gpu"]
