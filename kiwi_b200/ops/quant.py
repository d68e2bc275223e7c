"""1x128 block FP8 e4m3 quantisation of bf16 rows as a stand-alone op:
``quant_fp8(x) -> (codes float8_e4m3fn [T, H], fp32 scales [T, H / 128])``
with scale = amax / 448 per block (1 for an all-zero block).

CUDA tensors run the EP dispatch kernel's arithmetic in a kernel of its own
(``kiwi_b200._C.ops.quant_fp8``); CPU tensors run
:func:`kiwi_b200.models.moe.quant_fp8_codes`.  The two can differ by one code
where a value lies exactly between two e4m3 codes.
"""
import torch

from ..models import moe as _moe


def quant_fp8(x):
    """(codes, scales) of bf16 rows x [T, H], H a multiple of 128."""
    if not x.is_cuda:
        return _moe.quant_fp8_codes(x)
    from .. import native

    return native().ops.quant_fp8(x.to(torch.bfloat16).contiguous())


__all__ = ["quant_fp8"]
