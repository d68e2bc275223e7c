"""Drop-in name for code written against the reference's EP extension.

    import kiwi_b200.parallel.kiwi_ep_ext as kiwi_ep_ext
    op = kiwi_ep_ext.KiwiEpOp(device_id, world_size, hidden_dim, topk, num_experts_per_rank,
                              max_num_inp_token_per_rank, dispatch_dtype, combine_dtype)

Exposes the module-level API of the reference's ``kiwi_ep_ext``
(apps/ep/python/kiwi_ep_bindings.hip.cpp:580-640 of AMDResearch/kiwi):
``KiwiEpOp``, ``barrier``, ``get_rank``, ``get_nranks``,
``get_hca_name_for_gpu``, ``get_hca_name_for_current_gpu``,
``recommended_num_blocks``, ``recommended_runtime_defaults``.  The
reference's ``LciContext`` runtime guard becomes a no-op context manager that
initialises the process group from the launcher's environment (torchrun,
mpirun or srun variables).  ``CollectiveEpOp`` is the same operator contract
over NCCL all-to-all, for ranks that span nodes.
"""
from ..utils import dist as _dist
from .ep import (KiwiEpOp, barrier, get_hca_name_for_current_gpu, get_hca_name_for_gpu, get_nranks, get_rank,
                 recommended_num_blocks, recommended_runtime_defaults)
from .ep_collective import CollectiveEpOp


class LciContext:
    """Process-group guard in place of the reference's LCI runtime guard:
    construction initialises torch.distributed from the launcher's variables;
    usable as a context manager.  The device name argument is ignored."""

    def __init__(self, device_name=""):
        self.rank, self.nranks = _dist.init()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


__all__ = ["KiwiEpOp", "CollectiveEpOp", "LciContext", "barrier", "get_rank", "get_nranks", "get_hca_name_for_gpu",
           "get_hca_name_for_current_gpu", "recommended_num_blocks", "recommended_runtime_defaults"]
