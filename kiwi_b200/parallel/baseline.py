"""On-box baseline of the EP MoE layer: NCCL all-to-all + cuBLAS/CUTLASS grouped
GEMM through stock PyTorch (the path the fused kernels must beat).

Same routing, same dispatch format (1x128 FP8 or NVFP4, quantised with torch ops), same
bf16 expert FFN (``torch._grouped_mm``) and the same weights as
:class:`kiwi_b200.parallel.ep.ExpertParallelMoE`; the all-to-alls are
``torch.distributed.all_to_all_single`` over NCCL.  Not product code: it
exists to be measured against.
"""
import torch
import torch.distributed as dist
import torch.nn.functional as F

from ..models import moe as moe_model
from ..utils import dist as kdist


def _quant_fp8(x, block=128):
    t, h = x.shape
    xb = x.float().view(t, h // block, block)
    amax = xb.abs().amax(-1, keepdim=True)
    scale = torch.where(amax > 0, amax / moe_model.FP8_MAX, torch.ones_like(amax))
    q = (xb / scale).to(torch.float8_e4m3fn).view(t, h)
    return q, scale.view(t, h // block)


def _dequant_fp8(q, scale, block=128):
    t, h = q.shape
    return (q.float().view(t, h // block, block) * scale.view(t, h // block, 1)).view(t, h).to(torch.bfloat16)


def _grouped_mm(a, w, offs):
    """a [P, K] bf16, w [G, N, K] bf16, offs int32 [G] cumulative row ends -> [P, N]."""
    try:
        return torch._grouped_mm(a, w.transpose(-2, -1), offs=offs, out_dtype=torch.bfloat16)
    except Exception:
        out = torch.empty(a.shape[0], w.shape[1], dtype=torch.bfloat16, device=a.device)
        start = 0
        for g, end in enumerate(offs.tolist()):
            if end > start:
                out[start:end] = a[start:end] @ w[g].t()
            start = end
        return out


class NcclMoEBaseline:
    """The same MoE layer built from library calls, for the on-box baseline:
    torch top-k routing and block quantisation (1x128 FP8, or NVFP4 for an
    ``nvfp4`` config), NCCL all-to-all (``all_to_all_single``) of one packed
    record per (token, destination rank) -- row, scales, top-k ids and weights
    in one buffer, so one all-to-all per direction after the row-count
    exchange -- ``torch._grouped_mm`` for both expert GEMMs, one all-to-all of
    the per-(token, rank) partial sums back and a per-token sum.  The row
    counts must reach the host to size the uneven all-to-all (one
    synchronisation per step, as in every all_to_all_single EP layer).  Not
    product code: ``bench.py`` times it next to the fused layer."""
    def __init__(self, cfg, group=None):
        self.cfg = cfg
        self.group = group
        self.rank = kdist.rank(group)
        self.world = kdist.world_size(group)
        self.epr = cfg.num_experts // self.world
        dev = torch.device("cuda", torch.cuda.current_device())
        w13 = torch.empty(self.epr, 2 * cfg.ffn, cfg.hidden, dtype=torch.bfloat16, device=dev)
        w2 = torch.empty(self.epr, cfg.hidden, cfg.ffn, dtype=torch.bfloat16, device=dev)
        for j in range(self.epr):
            a, b, c = moe_model.expert_weights(cfg, self.rank * self.epr + j, dev)
            w13[j, :cfg.ffn] = a
            w13[j, cfg.ffn:] = b
            w2[j] = c
        self.w13, self.w2 = w13, w2

    def _a2a(self, out, inp, out_splits, in_splits):
        if self.world == 1:
            out.copy_(inp)
        else:
            dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def _quant(self, x):
        """(wire rows uint8 [T, B], scale bytes uint8 [T, S]) of bf16 rows."""
        if self.cfg.quant == "nvfp4":
            return moe_model.quant_nvfp4_codes(x)
        q, s = _quant_fp8(x)
        return q.view(torch.uint8), s.contiguous().view(torch.uint8).view(x.shape[0], -1)

    def _dequant(self, rows, scales):
        if self.cfg.quant == "nvfp4":
            return moe_model.dequant_nvfp4(rows, scales).to(torch.bfloat16)
        return _dequant_fp8(rows.view(torch.float8_e4m3fn), scales.contiguous().view(torch.float32))

    def forward(self, x, logits):
        cfg = self.cfg
        t, k = x.shape[0], cfg.topk
        v, idx = torch.topk(logits, k, dim=-1)
        w = torch.softmax(v, dim=-1)
        dest = idx // self.epr
        mask = torch.zeros(t, self.world, dtype=torch.bool, device=x.device)
        mask.scatter_(1, dest, True)
        _, t_of = mask.t().nonzero(as_tuple=True)              # (rank, token) pairs sorted by rank
        send_counts = mask.sum(0)
        q, s = self._quant(x)
        rb, sb = q.shape[1], s.shape[1]
        rec = torch.cat([q, s, idx.to(torch.int32).view(torch.uint8).view(t, 4 * k),
                         w.view(torch.uint8).view(t, 4 * k)], dim=1)[t_of]
        if self.world > 1:
            recv_counts = torch.empty_like(send_counts)
            dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        else:
            recv_counts = send_counts
        in_splits = send_counts.tolist()
        out_splits = recv_counts.tolist()
        n = sum(out_splits)
        got = torch.empty(n, rec.shape[1], dtype=torch.uint8, device=x.device)
        self._a2a(got, rec, out_splits, in_splits)
        rows = self._dequant(got[:, :rb], got[:, rb:rb + sb])
        ri = got[:, rb + sb:rb + sb + 4 * k].contiguous().view(torch.int32)
        rw = got[:, rb + sb + 4 * k:].contiguous().view(torch.float32)
        local = ri - self.rank * self.epr
        ok = (local >= 0) & (local < self.epr)
        row_id, slot = ok.nonzero(as_tuple=True)
        e = local[row_id, slot]
        order = torch.argsort(e, stable=True)
        row_id, slot, e = row_id[order], slot[order], e[order]
        counts = torch.bincount(e, minlength=self.epr)
        offs = torch.cumsum(counts, 0).to(torch.int32)
        a = rows[row_id]
        h1 = _grouped_mm(a, self.w13, offs)
        hdn = (F.silu(h1[:, :cfg.ffn].float()) * h1[:, cfg.ffn:].float()).to(torch.bfloat16)
        y = _grouped_mm(hdn, self.w2, offs).float() * rw[row_id, slot][:, None]
        back = torch.zeros(n, cfg.hidden, dtype=torch.float32, device=x.device)
        back.index_add_(0, row_id, y)
        back = back.to(torch.bfloat16)
        ret = torch.empty(t_of.shape[0], cfg.hidden, dtype=torch.bfloat16, device=x.device)
        self._a2a(ret, back, in_splits, out_splits)
        out = torch.zeros(t, cfg.hidden, dtype=torch.float32, device=x.device)
        out.index_add_(0, t_of, ret.float())
        return out.to(torch.bfloat16)

    __call__ = forward
