"""kiwi_b200.parallel: the multi-GPU layers (each a module, imported on use).

* :mod:`.p2p`            symmetric heap over NVLink, device put / get / signal, NVLS, copy-engine puts
* :mod:`.collectives`    device all-to-all, cross-rank barrier and grid barrier with bounded waits
* :mod:`.ep`             the fused expert-parallel MoE layer (``ExpertParallelMoE``) and the MORI-style
                         ``KiwiEpOp`` transport, one NVSwitch domain
* :mod:`.ep_collective`  ``CollectiveEpOp`` / ``CollectiveMoE``: the same contract and layer over
                         torch.distributed all-to-all, for ranks on several nodes (or gloo on CPU)
* :mod:`.kiwi_ep_ext`    the reference extension's module-level API under its name
* :mod:`.baseline`       the NCCL all-to-all + grouped-GEMM baseline of the benchmarks
"""
