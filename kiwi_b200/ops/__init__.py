"""kiwi_b200.ops: compute ops.

* :class:`GroupedGemm` / :func:`grouped_gemm`: grouped BF16 GEMM (sm_100a
  tcgen05 kernel for CUDA tensors; fp32 reference for CPU tensors) with the
  fused SwiGLU and per-row-scale epilogues.
* :class:`ExpertFFN`: the local experts' SwiGLU FFN on expert-sorted rows.
* :func:`grouped_gemm_reference`: the fp32 restatement the kernel is tested against.
* :func:`block_weights` / :func:`unblock_weights`: the blocked weight layout
  (one contiguous 256 x 64 box per TMA load) and back.
* :func:`copy_rows` / :func:`accumulate_rows`: the pack / unpack / copy and
  top-k accumulate row patterns of EP dispatch and combine as stand-alone
  kernels (``benchmarks/bench_ep_copy.py`` measures them against HBM).

* :func:`route_topk`: top-k routing with the softmax over the selected logits
  (the EP layer's routing kernel).
* :func:`quant_fp8` / :func:`quant_nvfp4`: 1x128 FP8 and NVFP4 quantisation
  with the dispatch kernel's arithmetic (its wire bytes).

Inside the NVLink EP layer, routing and FP8 / NVFP4 quantisation run fused
into its own kernels (:mod:`kiwi_b200.parallel.ep`); the fp32 references are
in :mod:`kiwi_b200.models.moe`.
"""
from .grouped_gemm import (ExpertFFN, GroupedGemm, block_weights, grouped_gemm, grouped_gemm_reference,
                           unblock_weights)
from .quant import quant_fp8, quant_nvfp4
from .routing import route_topk
from .rows import accumulate_rows, check_error, copy_rows

__all__ = ["ExpertFFN", "GroupedGemm", "block_weights", "unblock_weights", "grouped_gemm", "grouped_gemm_reference",
           "accumulate_rows", "check_error", "copy_rows", "quant_fp8", "quant_nvfp4", "route_topk"]
