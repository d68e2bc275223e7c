"""Block quantisation of bf16 rows as stand-alone ops, with the EP dispatch
kernel's arithmetic:

* ``quant_fp8(x) -> (codes float8_e4m3fn [T, H], fp32 scales [T, H / 128])``,
  1x128 blocks, scale = amax / 448 per block (1 for an all-zero block);
* ``quant_nvfp4(x) -> (packed e2m1 codes uint8 [T, H / 2], scale bytes uint8
  [T, S])``, the NVLink dispatch's NVFP4 wire bytes: an fp32 row scale
  amax / (448 * 6), then one e4m3 scale per 16 elements relative to it, zero
  padding to 16 bytes.

CUDA tensors run the dispatch kernel's arithmetic in kernels of their own
(``kiwi_b200._C.ops.quant_fp8`` / ``quant_nvfp4``), so a transport that
quantises with them carries the same bytes as the fused dispatch; CPU tensors
run :func:`kiwi_b200.models.moe.quant_fp8_codes` /
:func:`kiwi_b200.models.moe.quant_nvfp4_codes`, which can differ from the
kernel by one code where a value lies exactly between two codes.
"""
import torch

from ..models import moe as _moe


def quant_fp8(x):
    """(codes, scales) of bf16 rows x [T, H], H a multiple of 128."""
    if not x.is_cuda:
        return _moe.quant_fp8_codes(x)
    from .. import native

    return native().ops.quant_fp8(x.to(torch.bfloat16).contiguous())


def quant_nvfp4(x):
    """(packed codes, scale bytes) of bf16 rows x [T, H], H a multiple of 16."""
    if not x.is_cuda:
        return _moe.quant_nvfp4_codes(x)
    from .. import native

    return native().ops.quant_nvfp4(x.to(torch.bfloat16).contiguous())


__all__ = ["quant_fp8", "quant_nvfp4"]
