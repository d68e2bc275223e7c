"""kiwi_b200.ops: compute ops.

* :class:`GroupedGemm` / :func:`grouped_gemm`: grouped BF16 GEMM (sm_100a
  tcgen05 kernel for CUDA tensors; fp32 reference for CPU tensors) with the
  fused SwiGLU and per-row-scale epilogues.
* :class:`ExpertFFN`: the local experts' SwiGLU FFN on expert-sorted rows.
* :func:`grouped_gemm_reference`: the fp32 restatement the kernel is tested against.

Routing and FP8 / NVFP4 quantisation run fused into the EP dispatch kernel
(:mod:`kiwi_b200.parallel.ep`); their fp32 references are in
:mod:`kiwi_b200.models.moe`.
"""
from .grouped_gemm import ExpertFFN, GroupedGemm, grouped_gemm, grouped_gemm_reference

__all__ = ["ExpertFFN", "GroupedGemm", "grouped_gemm", "grouped_gemm_reference"]
