"""kiwi_b200: kernel-initiated invocations, NVLink P2P and expert-parallel MoE for B200.

Layers (each a sub-package or module):

* ``kiwi_b200.queue``    GPU<->host rings in mapped pinned memory (native: ``include/kiwi/queue``)
* ``kiwi_b200.invoke``   callbacks a running kernel calls on the host (native: ``include/kiwi/invoke``)
* ``kiwi_b200.parallel`` NVLink symmetric heap, P2P put/get/signal, EP dispatch/combine
* ``kiwi_b200.ops``      grouped GEMM and expert FFN (sm_100a tcgen05 kernel; fp32 reference on CPU)
* ``kiwi_b200.models``   the MoE layer built from them, plus fp32 reference implementations
* ``kiwi_b200.utils``    timing, clocks, topology, build helpers
"""
from ._native import load as _load_native

__version__ = "0.1.0"


def native():
    """The native extension module (raises ImportError if it is not built)."""
    return _load_native()
