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
    """CPUs local to CUDA device `device` that this process may run on."""
    local = set(_load().topology.gpu_local_cpus(int(device)))
    allowed = os.sched_getaffinity(0)
    return sorted(local & allowed)


def bind_process_to_gpu(device):
    """Restricts this process to `device`'s local CPUs; returns them (empty list,
    and nothing changed, when the node's CPUs are unknown or not allowed)."""
    cpus = gpu_local_cpus(device)
    if cpus:
        os.sched_setaffinity(0, cpus)
    return cpus


__all__ = ["gpu_local_cpus", "bind_process_to_gpu"]
