"""kiwi_b200.parallel.ep: expert-parallel MoE over NVLink on B200.

:class:`ExpertParallelMoE` is one rank's share of a MoE layer whose experts are
sharded contiguously over the ranks of ``group`` (expert e lives on rank
``e // (num_experts // world)``, as in the reference, apps/ep/ep_config.hpp:203-204
of AMDResearch/kiwi).  ``forward(x, router_logits)`` runs, on the current CUDA
stream and without host synchronisation:

1. routing: top-k + softmax over the selected logits;
2. dispatch: 1x128 FP8 (or NVFP4 / bf16) quantisation fused with 16-byte
   NVLink stores into every destination rank's receive slots, deduplicated
   per destination rank, one release flag per source rank;
3. receive: per-expert counts, expert-major layout, dequantisation to bf16;
4. experts: tcgen05 grouped GEMM (SwiGLU fused) then grouped GEMM (routing
   weight fused), bf16 compute with fp32 accumulation;
5. combine: each slot's weighted expert rows summed and stored back into the
   token owner's combine slots over NVLink, then reduced per token.

``stage(...)`` methods expose the phases separately for profiling, and
:class:`EpDispatchCombine` gives the reference's transport-only
dispatch/combine contract (rows in, rows out).
"""
import torch

from .._native import load as _load
from ..models import moe as moe_model
from ..utils import dist as kdist
from .p2p import SymmetricHeap

_C = _load()

QUANTS = ("fp8", "nvfp4", "none")


def layer_config(cfg, rank, world, max_tokens=None):
    """The native EpConfig (dict) of a MoEConfig on `world` ranks."""
    d = dict(world=world, rank=rank, hidden=cfg.hidden, num_experts=cfg.num_experts, topk=cfg.topk,
             max_tokens=max_tokens or cfg.tokens_per_rank, quant=cfg.quant)
    return _C.ep.finalize_config(d)


class ExpertParallelMoE:
    """One rank's expert-parallel MoE layer (collective constructor)."""

    def __init__(self, cfg, group=None, max_tokens=None, weights=None, timeout_s=5.0, heap=None):
        if cfg.quant not in QUANTS:
            raise ValueError(f"quant must be one of {QUANTS}")
        self.cfg = cfg
        self.group = group
        self.rank = kdist.rank(group)
        self.world = kdist.world_size(group)
        if cfg.num_experts % self.world:
            raise ValueError("num_experts must be divisible by the world size")
        self.max_tokens = max_tokens or cfg.tokens_per_rank
        self.layout = layer_config(cfg, self.rank, self.world, self.max_tokens)
        self.heap = heap or SymmetricHeap(self.layout["heap_bytes"], group)
        dev = torch.device("cuda", torch.cuda.current_device())
        if weights is None:
            weights = moe_model.local_expert_weights(cfg, self.rank, self.world, dev)
        self.w13, self.w2 = weights
        self._layer = _C.ep.MoeLayer(self.heap.native, self.layout, cfg.ffn, self.w13, self.w2,
                                     int(timeout_s * 1e9))
        k = cfg.topk
        self._idx = torch.empty(self.max_tokens, k, dtype=torch.int32, device=dev)
        self._w = torch.empty(self.max_tokens, k, dtype=torch.float32, device=dev)
        self._out = torch.empty(self.max_tokens, cfg.hidden, dtype=torch.bfloat16, device=dev)

    # -- the layer -------------------------------------------------------------
    def route(self, router_logits):
        t = router_logits.shape[0]
        idx, w = self._idx[:t], self._w[:t]
        self._layer.route(router_logits.contiguous(), idx, w)
        return idx, w

    def forward(self, x, router_logits, out=None):
        """x [T, hidden] bf16, router_logits [T, num_experts] fp32 -> [T, hidden] bf16.
        The returned tensor is operator-owned unless `out` is given."""
        t = x.shape[0]
        idx, w = self.route(router_logits)
        out = self._out[:t] if out is None else out
        self._layer.forward(x.contiguous(), idx, w, out)
        return out

    __call__ = forward

    def forward_routed(self, x, idx, w, out=None):
        """Same layer with precomputed routing (idx int32 [T, k], w fp32 [T, k])."""
        out = self._out[:x.shape[0]] if out is None else out
        self._layer.forward(x.contiguous(), idx.contiguous(), w.contiguous(), out)
        return out

    # -- stages (profiling) ------------------------------------------------------
    def stage_dispatch(self, x, idx, w):
        self._layer.dispatch(x, idx, w)

    def stage_receive(self):
        self._layer.receive()

    def stage_experts(self):
        self._layer.experts()

    def stage_combine(self, idx, out):
        self._layer.combine(idx, out)

    # -- diagnostics --------------------------------------------------------------
    def check(self):
        """Raises if a device-side wait timed out or a capacity check failed."""
        code, site, info, rank, gemm = self._layer.error()
        if code or gemm:
            raise RuntimeError(f"kiwi ep error: code={code} site={site} info={info} rank={rank} gemm={gemm}")

    @property
    def expert_counts(self):
        return self._layer.expert_counts

    @property
    def native(self):
        return self._layer


class EpDispatchCombine:
    """Transport-only dispatch / combine with the reference's contract
    (apps/ep/python/kiwi_ep_bindings.hip.cpp:289-373 of AMDResearch/kiwi):
    ``dispatch(x, weights, indices)`` returns the rows received on this rank
    (expert-major, with their source slot, routing weight and expert id) and
    ``combine(expert_rows)`` sends each row back to its token's rank and sums
    them per token.  Built on the same kernels as ExpertParallelMoE with the
    expert FFN replaced by the caller's computation."""

    def __init__(self, hidden, num_experts, topk, max_tokens, quant="none", group=None, timeout_s=5.0):
        cfg = moe_model.MoEConfig(hidden=hidden, ffn=256, num_experts=num_experts, topk=topk,
                                  tokens_per_rank=max_tokens, quant=quant, name="transport")
        world = kdist.world_size(group)
        dev = torch.device("cuda", torch.cuda.current_device())
        epr = num_experts // world
        w13 = torch.zeros(epr * 2 * cfg.ffn, hidden, dtype=torch.bfloat16, device=dev)
        w2 = torch.zeros(epr * hidden, cfg.ffn, dtype=torch.bfloat16, device=dev)
        self.moe = ExpertParallelMoE(cfg, group, max_tokens, weights=(w13, w2), timeout_s=timeout_s)
        self._idx = None

    def dispatch(self, x, weights, indices):
        """Returns (rows [R, hidden] bf16, counts per local expert, slot of each row, weight of each row)."""
        self._idx = indices.contiguous()
        self.moe.stage_dispatch(x.contiguous(), self._idx, weights.contiguous())
        self.moe.stage_receive()
        layer = self.moe.native
        return layer.expert_input, layer.expert_counts, layer.pair_slot, layer.pair_weight

    def combine(self, expert_rows, out=None):
        """expert_rows: [R, hidden] bf16 outputs, one per dispatched row (already
        weighted by the caller if it wants a weighted sum)."""
        layer = self.moe.native
        y = layer.expert_output
        y[:expert_rows.shape[0]].copy_(expert_rows)
        t = self._idx.shape[0]
        out = torch.empty(t, y.shape[1], dtype=torch.bfloat16, device=y.device) if out is None else out
        self.moe.stage_combine(self._idx, out)
        return out


__all__ = ["ExpertParallelMoE", "EpDispatchCombine", "layer_config"]
