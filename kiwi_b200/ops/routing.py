"""Top-k routing as a stand-alone op: each token's ``topk`` largest router
logits and the softmax over them.

CUDA tensors run the EP layer's routing kernel (``kiwi_b200._C.ops.route_topk``,
one warp per token, up to 1024 experts and top-16); CPU tensors run
:func:`kiwi_b200.models.moe.route_reference`.  Returns ``(idx int32 [T, k],
weights fp32 [T, k])``, experts in descending logit order.
"""
import torch

from ..models import moe as _moe


def route_topk(logits, topk):
    """(expert ids, routing weights) of each token; see the module docstring."""
    if not logits.is_cuda:
        return _moe.route_reference(logits, topk)
    from .. import native

    return native().ops.route_topk(logits.float().contiguous(), int(topk))


__all__ = ["route_topk"]
