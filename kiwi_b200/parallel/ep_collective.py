"""KiwiEpOp's dispatch / combine contract over torch.distributed all-to-all.

``CollectiveEpOp`` has the same constructor arguments, methods and return
values as :class:`kiwi_b200.parallel.ep.KiwiEpOp`, but moves the rows with
``all_to_all_single`` (NCCL between GPUs, gloo between CPU processes) instead
of NVLink stores into a symmetric heap.  It is the way to run the transport on
ranks that do not share one NVSwitch domain (several nodes), which
:class:`~kiwi_b200.parallel.ep.KiwiEpOp` does not span, and it runs on CPU
processes too.  The caller chooses it explicitly; nothing switches between the
two.  (The reference spans nodes with LCI RDMA through CPU proxies,
apps/ep/dispatch.hip.cpp and apps/ep/comm of AMDResearch/kiwi.)

Semantics, as KiwiEpOp:

* ``dispatch(input, weights, scales, indices)`` returns ``(out, out_weights,
  out_scales, out_indices, recv_count)``: one row per (source rank, token) that
  routes at least one of its top-k experts to this rank, in (source rank,
  token) order; ``out`` in the wire format (bf16; float8_e4m3fn with fp32
  1x128 scales in ``out_scales``; or NVFP4 as the NVLink op carries it: packed
  e2m1 bytes [n, hidden / 2] and, in ``out_scales``, an fp32 row scale then
  e4m3 block scales per 16 elements, padded to 16 bytes), ``out_weights`` /
  ``out_indices`` the token's
  full top-k weights and global expert ids.  bf16 input is quantised here
  (``scales`` ignored); float8_e4m3fn input with per-token fp32 ``scales``
  [T, S], or packed FP4 input (uint8 / float4_e2m1fn_x2 [T, hidden / 2]) with
  per-token scales of any dtype (the reference's pre-quantised contract),
  travels unchanged (FP4 scales come back as their bytes).
* ``combine(input, weights, indices, out)`` returns ``(out, out_weights)``: row i of
  ``input`` goes back to the rank and token it came from, and each token's rows
  are summed in fp32 (no routing weights, as MORI); tokens routed nowhere get
  zeros.  Rows travel and the result is returned in ``combine_dtype``: bf16,
  float32, float8_e4m3fn or float4_e2m1fn_x2 (codes without scales, the sum
  re-quantised with saturation; FP4 rows are hidden / 2 bytes, element 2i in
  the low nibble), as the reference also accepts.  With ``weights`` (fp32
  [rows, topk]) the rows' weights travel back and ``out_weights`` [T, topk]
  holds each token's sum; otherwise it is None.
* ``get_dispatch_src_token_pos()`` encodes each received row's source as
  ``src_rank * (world * max_tokens) + token`` and ``decode_send_flat_idx``
  inverts it.

Per dispatch there are two all-to-alls (the per-rank row counts, then one
record per row holding the row, its weights, ids, source token and scales),
and one per combine; every rank must call dispatch and combine in the same
order.
"""
import math

import torch
import torch.distributed as dist

from ..models import moe as moe_model
from ..ops import ExpertFFN, quant_fp8, quant_nvfp4, route_topk
from ..utils import dist as kdist

_FORMATS = {"none": "none", "fp8": "fp8", "fp4": "nvfp4", "nvfp4": "nvfp4"}
_DTYPES = {torch.bfloat16: "none", torch.float8_e4m3fn: "fp8"}
_FP4 = torch.float4_e2m1fn_x2
_COMBINE_DTYPES = (torch.bfloat16, torch.float32, torch.float8_e4m3fn, _FP4)
_FP8_MAX = 448.0


def _to_combine_dtype(x, dtype):
    """x in `dtype`; FP8 saturates at +-448 (e4m3fn has no infinity); FP4
    (e2m1, two per byte, so [rows, hidden / 2]) rounds to nearest-even and
    saturates at +-6.  FP4 input already packed passes through."""
    if dtype == _FP4:
        if x.dtype in (_FP4, torch.uint8):
            return x.view(_FP4)
        return moe_model.fp4_pack(moe_model.fp4_codes(x)).view(_FP4)
    if dtype == torch.float8_e4m3fn and x.dtype != dtype:
        return x.float().clamp(-_FP8_MAX, _FP8_MAX).to(dtype)
    return x.to(dtype)


def _to_float(x):
    return moe_model.fp4_unpack(x) if x.dtype == _FP4 else x.float()


class CollectiveEpOp:
    """KiwiEpOp's transport contract over torch.distributed all-to-all (see the module docstring)."""

    def __init__(self, device_id=None, world_size=None, hidden_dim=None, topk=None, num_experts_per_rank=None,
                 max_num_inp_token_per_rank=None, dispatch_dtype=torch.bfloat16, combine_dtype=torch.bfloat16,
                 num_blocks=None, num_proxy_threads=4, dispatch_elem_size=-1, dispatch_scale_dim=0,
                 dispatch_scale_type_size=0, combine_scale_dim=0, combine_scale_type_size=0,
                 dispatch_scale_dtype=None, device_name="", dispatch_quant_format="none",
                 combine_quant_format="none", queue_capacity=2048, rcomp_backend="auto", *, group=None,
                 device=None):
        """Arguments as KiwiEpOp (the reference's names and order).  The launch
        and proxy arguments (num_blocks, num_proxy_threads, queue_capacity,
        device_name, rcomp_backend) have no meaning for an all-to-all transport
        and change nothing; combine scales are not carried and raise."""
        missing = [n for n, v in (("hidden_dim", hidden_dim), ("topk", topk),
                                  ("num_experts_per_rank", num_experts_per_rank),
                                  ("max_num_inp_token_per_rank", max_num_inp_token_per_rank)) if v is None]
        if missing:
            raise TypeError("CollectiveEpOp missing required arguments: " + ", ".join(missing))
        if int(combine_scale_dim) or int(combine_scale_type_size):
            raise ValueError("combine scales are not carried (combine_scale_dim / combine_scale_type_size must be 0)")
        cfmt = str(combine_quant_format).lower()
        if cfmt == "fp8" and combine_dtype in (torch.uint8, torch.float8_e4m3fn):
            combine_dtype = torch.float8_e4m3fn
        elif cfmt == "fp4" and combine_dtype in (torch.uint8, _FP4):
            combine_dtype = _FP4
        elif cfmt != "none" or combine_dtype not in _COMBINE_DTYPES:
            raise ValueError("combine_dtype must be torch.bfloat16, torch.float32, torch.float8_e4m3fn or "
                             "torch.float4_e2m1fn_x2 (or uint8 with combine_quant_format 'fp8' / 'fp4')")
        self._combine_dtype = combine_dtype
        if combine_dtype == _FP4 and hidden_dim % 2:
            raise ValueError("FP4 combine needs an even hidden_dim (two elements per byte)")
        fmt = str(dispatch_quant_format).lower()
        if fmt not in _FORMATS:
            raise ValueError(f"unsupported dispatch_quant_format {dispatch_quant_format!r} (none, fp8 or fp4)")
        quant = _FORMATS[fmt] if fmt != "none" else _DTYPES.get(dispatch_dtype)
        if quant is None:
            raise ValueError(f"unsupported dispatch_dtype {dispatch_dtype}")
        if hidden_dim % 128 and quant == "fp8":
            raise ValueError("FP8 dispatch needs hidden_dim to be a multiple of 128")
        if hidden_dim % 16 and quant == "nvfp4":
            raise ValueError("NVFP4 dispatch needs hidden_dim to be a multiple of 16")
        self.group = group
        self.rank = kdist.rank(group)
        self.world_size = kdist.world_size(group)
        if world_size is not None and int(world_size) != self.world_size:
            raise ValueError(f"world_size {world_size} differs from the process group's {self.world_size}")
        if device is None:
            if device_id is not None:
                torch.cuda.set_device(int(device_id))
                device = torch.device("cuda", int(device_id))
            elif torch.cuda.is_available() and (not dist.is_initialized() or dist.get_backend(group) == "nccl"):
                device = torch.device("cuda", torch.cuda.current_device())
            else:
                device = torch.device("cpu")
        self.device = torch.device(device)
        self.hidden_dim = int(hidden_dim)
        self.topk = int(topk)
        self.experts_per_rank = int(num_experts_per_rank)
        self.max_tokens = int(max_num_inp_token_per_rank)
        self._quant = quant
        self._send_counts = None
        self._recv_counts = None
        self._send_tokens = None
        self._src_pos = None
        self._last_tokens = 0
        self._out = None

    # -- helpers ------------------------------------------------------------------
    def _a2a(self, send, send_counts, recv_counts):
        """all_to_all_single of the rows of `send` (first dimension split by rank)."""
        shape = (int(sum(recv_counts)),) + tuple(send.shape[1:])
        recv = torch.empty(shape, dtype=send.dtype, device=send.device)
        if self.world_size == 1:
            recv.copy_(send)
            return recv
        dist.all_to_all_single(recv, send.contiguous(), output_split_sizes=list(recv_counts),
                               input_split_sizes=list(send_counts), group=self.group)
        return recv

    def _wire(self, t):
        """A payload tensor as bytes (all_to_all needs types every backend carries)."""
        row_bytes = t.element_size() * math.prod(t.shape[1:])
        return t.contiguous().view(torch.uint8).view(t.shape[0], row_bytes)

    @staticmethod
    def _unwire(recv, like):
        """Splits received records back into tensors of the dtypes and widths of `like`."""
        out, off, n = [], 0, recv.shape[0]
        for f in like:
            nb = f.element_size() * math.prod(f.shape[1:])
            out.append(recv[:, off:off + nb].contiguous().view(f.dtype).view(n, *f.shape[1:]))
            off += nb
        return out

    # -- the contract ---------------------------------------------------------------
    def dispatch(self, input, weights, scales=None, indices=None, **_launch_kwargs):
        """See the module docstring; collective over the group."""
        x = input.to(self.device)
        t = x.shape[0]
        if t > self.max_tokens:
            raise ValueError("more tokens than max_num_inp_token_per_rank")
        idx = indices.to(self.device, torch.int64)
        w = weights.to(self.device, torch.float32)
        if t and (int(idx.min()) < 0 or int(idx.max()) >= self.world_size * self.experts_per_rank):
            raise ValueError("expert indices must lie in [0, world_size * num_experts_per_rank)")
        dest = idx // self.experts_per_rank                                           # [T, k]
        onehot = torch.zeros(t, self.world_size, dtype=torch.bool, device=self.device)
        if t:
            onehot.scatter_(1, dest, True)
        pairs = onehot.t().nonzero()                                                   # (dest, token), dest-major
        order_dest, order_tok = pairs[:, 0], pairs[:, 1]
        send_counts = torch.bincount(order_dest, minlength=self.world_size)
        recv_counts = self._a2a(send_counts.view(-1, 1), [1] * self.world_size, [1] * self.world_size).view(-1)
        send_counts, recv_counts = send_counts.tolist(), recv_counts.tolist()
        if x.dtype == torch.float8_e4m3fn:
            # Pre-quantised by the caller (the reference's dispatch contract): codes
            # and the caller's per-token scales travel unchanged.
            if self._quant != "fp8" or scales is None or scales.shape[0] != t:
                raise ValueError("FP8 input needs an FP8 op and per-token scales [T, S]")
            rows, row_scales = x[order_tok], scales.to(self.device, torch.float32).reshape(t, -1)[order_tok]
        elif x.dtype in (torch.uint8, _FP4):
            # Packed e2m1 codes [T, hidden / 2] pre-quantised by the caller: codes and
            # the caller's per-token scale bytes travel unchanged.
            if self._quant != "nvfp4" or scales is None or scales.shape[0] != t or x.shape[1] * 2 != self.hidden_dim:
                raise ValueError("packed FP4 input needs an NVFP4 op, [T, hidden / 2] codes and per-token scales")
            rows = x.view(torch.uint8)[order_tok]
            row_scales = scales.to(self.device).contiguous().view(torch.uint8).reshape(t, -1)[order_tok]
        elif self._quant == "fp8":
            codes, sc = quant_fp8(x)  # the dispatch kernel's arithmetic on CUDA tensors
            rows, row_scales = codes[order_tok], sc[order_tok]
        elif self._quant == "nvfp4":
            codes, sc = quant_nvfp4(x)  # the NVLink op's wire bytes (its kernel's arithmetic on CUDA)
            rows, row_scales = codes[order_tok], sc[order_tok]
        else:
            rows, row_scales = x.to(torch.bfloat16)[order_tok], None
        # One record per row, [row | weights | ids | source token | scales], so
        # the payload crosses in a single all-to-all.
        fields = [rows, w[order_tok], idx.to(torch.int32)[order_tok], order_tok.to(torch.int32).view(-1, 1)]
        if row_scales is not None:
            fields.append(row_scales)
        recv = self._a2a(torch.cat([self._wire(f) for f in fields], dim=1), send_counts, recv_counts)
        out_rows, out_w, out_idx, src_tok, *rest = self._unwire(recv, fields)
        out_sc = rest[0] if rest else None
        src_tok = src_tok.view(-1)
        n = int(sum(recv_counts))
        src_rank = torch.repeat_interleave(torch.arange(self.world_size, device=self.device),
                                           torch.tensor(recv_counts, device=self.device))
        self._src_pos = src_rank.to(torch.int64) * self.max_num_tokens_to_send() + src_tok.to(torch.int64)
        self._send_counts, self._recv_counts, self._send_tokens = send_counts, recv_counts, order_tok
        self._last_tokens = t
        count = torch.tensor([n], dtype=torch.int32, device=self.device)
        return out_rows, out_w, out_sc, out_idx, count

    dispatch_send = dispatch

    def dispatch_recv(self, **_kwargs):
        """dispatch() already completes the receive (kept for call-shape parity)."""

    def combine(self, input, weights=None, indices=None, out=None, **_launch_kwargs):
        """See the module docstring; collective over the group.  With
        ``weights`` (fp32 [rows, topk]) each row's weights travel back with it
        and the second return value holds each token's sum of them."""
        if self._send_counts is None:
            raise RuntimeError("combine needs a prior dispatch")
        n = int(sum(self._recv_counts))
        rows = _to_combine_dtype(input[:n].to(self.device), self._combine_dtype)
        fields = [rows]
        if weights is not None:
            fields.append(weights[:n].to(self.device, torch.float32).reshape(n, self.topk))
        back = self._a2a(torch.cat([self._wire(f) for f in fields], dim=1), self._recv_counts, self._send_counts)
        parts = self._unwire(back, fields)                                          # (dest, token) order
        t = self._last_tokens
        acc = torch.zeros(t, self.hidden_dim, dtype=torch.float32, device=self.device)
        if back.shape[0]:
            acc.index_add_(0, self._send_tokens, _to_float(parts[0]))
        if out is None:
            out = torch.empty(t, self._combine_cols(), dtype=self._combine_dtype, device=self.device)
        res = _to_combine_dtype(acc, out.dtype)
        if out.dtype == _FP4:  # copy_ has no FP4 kernel: move the bytes
            out[:t].view(torch.uint8).copy_(res.view(torch.uint8))
        else:
            out[:t].copy_(res)
        out_w = None
        if weights is not None:
            out_w = torch.zeros(t, self.topk, dtype=torch.float32, device=self.device)
            if back.shape[0]:
                out_w.index_add_(0, self._send_tokens, parts[1])
        self._out, self._out_w = out, out_w
        return out, out_w

    combine_send = combine

    def _combine_cols(self):
        """Columns of a combine row: hidden, or hidden / 2 bytes for FP4."""
        return self.hidden_dim // 2 if self._combine_dtype == _FP4 else self.hidden_dim

    def combine_recv(self, **_kwargs):
        return ((self._out[:self._last_tokens] if self._out is not None else None),
                getattr(self, "_out_w", None))

    def reset(self):
        """Ends the current round (nothing to clear between rounds)."""
        self._last_tokens = 0

    # -- accessors of the reference op -------------------------------------------
    def max_num_tokens_to_recv(self):
        return self.world_size * self.max_tokens

    def max_num_tokens_to_recv_per_rank(self):
        return self.max_tokens

    def max_num_tokens_to_send(self):
        return self.world_size * self.max_tokens

    def max_num_tokens_to_send_per_rank(self):
        return self.max_tokens

    def decode_send_flat_idx(self, flat_idx):
        """(source rank, source token) of a position from get_dispatch_src_token_pos()."""
        stride = self.max_num_tokens_to_send()
        return int(flat_idx) // stride, int(flat_idx) % stride

    def get_dispatch_src_token_pos(self):
        """Source position of each row the last dispatch received (see decode_send_flat_idx)."""
        return self._src_pos if self._src_pos is not None else torch.empty(0, dtype=torch.int64)

    def get_registered_combine_input_buffer(self, combine_dtype=None, hidden_dim=-1):
        """Operator-owned [max_num_tokens_to_recv(), hidden] buffer in the
        combine dtype, for expert outputs handed to combine() without a copy."""
        dt = self._combine_dtype if combine_dtype is None else combine_dtype
        if dt != self._combine_dtype:
            raise ValueError("combine_dtype must be the op's combine dtype")
        if hidden_dim > 0 and hidden_dim != self.hidden_dim:
            raise ValueError("get_registered_combine_input_buffer hidden_dim must match the configured hidden_dim")
        buf = getattr(self, "_combine_in", None)
        if buf is None:
            buf = self._combine_in = torch.empty(self.max_num_tokens_to_recv(), self._combine_cols(), dtype=dt,
                                                 device=self.device)
        return buf

    def launch_policy(self, num_tokens):
        return {"num_tokens": int(num_tokens), "transport": "torch.distributed all_to_all",
                "backend": dist.get_backend(self.group) if dist.is_initialized() else "none"}

    def check(self):
        """Nothing to check: errors surface as exceptions of the collectives."""


class CollectiveMoE:
    """One rank's expert-parallel MoE layer over :class:`CollectiveEpOp`.

    The same layer as :class:`kiwi_b200.parallel.ep.ExpertParallelMoE` (top-k
    softmax routing, dispatch in ``cfg.quant`` = "none", "fp8" or "nvfp4", each local
    expert's SwiGLU FFN, routing-weighted sum over the top-k experts), for ranks
    that do not share one NVSwitch domain: rows move with all-to-all, and each
    rank sums the contributions of its own experts to a received token before
    the token goes back, so one row per (token, destination rank) travels each
    way.  The experts run :class:`kiwi_b200.ops.ExpertFFN` (the tcgen05 grouped
    GEMM on CUDA tensors, its fp32 reference in CPU processes).  Collective:
    every rank of the group calls forward in the same order."""

    def __init__(self, cfg, group=None, max_tokens=None, weights=None, device=None, combine_dtype=torch.bfloat16):
        if cfg.quant not in ("none", "fp8", "nvfp4"):
            raise ValueError("CollectiveMoE carries bf16 ('none'), FP8 or NVFP4 rows")
        world = kdist.world_size(group)
        if cfg.num_experts % world:
            raise ValueError("num_experts must be divisible by the world size")
        self.cfg = cfg
        self.max_tokens = int(max_tokens or cfg.tokens_per_rank)
        self.experts_per_rank = cfg.num_experts // world
        self.op = CollectiveEpOp(hidden_dim=cfg.hidden, topk=cfg.topk, num_experts_per_rank=self.experts_per_rank,
                                 max_num_inp_token_per_rank=self.max_tokens, combine_dtype=combine_dtype,
                                 group=group, dispatch_quant_format=cfg.quant, device=device)
        self.device, self.rank, self.world = self.op.device, self.op.rank, self.op.world_size
        if weights is None:
            weights = moe_model.local_expert_weights(cfg, self.rank, self.world, self.device)
        max_pairs = self.world * self.max_tokens * min(cfg.topk, self.experts_per_rank)
        self.experts = ExpertFFN(weights[0], weights[1], self.experts_per_rank, max_pairs)
        # The expert GEMMs' own weights (on CUDA, blocked copies of the row-major inputs).
        self.w13, self.w2 = self.experts.gemm1.b, self.experts.gemm2.b
        self._scale = torch.zeros(max(max_pairs, 1), dtype=torch.float32, device=self.device)

    def forward(self, x, router_logits):
        """x [T, hidden] bf16, router_logits [T, num_experts] -> [T, hidden] (combine dtype)."""
        idx, w = route_topk(router_logits.to(self.device), self.cfg.topk)
        return self.forward_routed(x, idx, w)

    __call__ = forward

    def forward_routed(self, x, idx, w):
        """Same layer with precomputed routing (idx [T, k] global expert ids, w [T, k])."""
        rows, rw, scales, ridx, _ = self.op.dispatch(x, w, None, idx)
        n, h = rows.shape
        if self.cfg.quant == "nvfp4":  # e2m1 codes x block scales -> operand rows
            h = self.cfg.hidden
            rows = moe_model.dequant_nvfp4(rows, scales)
        elif scales is not None:  # FP8 codes x 1x128 scales -> operand rows
            rows = (rows.float().view(n, h // 128, 128) * scales.view(n, -1, 1)).view(n, h)
        local = ridx.long() - self.rank * self.experts_per_rank
        r, s = ((local >= 0) & (local < self.experts_per_rank)).nonzero(as_tuple=True)
        e = local[r, s]
        order = torch.argsort(e, stable=True)
        r, s, e = r[order], s[order], e[order]
        p = r.numel()
        counts = torch.bincount(e, minlength=self.experts_per_rank).to(torch.int32)
        self.experts.input_buffer()[:p].copy_(rows[r])
        self._scale[:p].copy_(rw[r, s])
        y = self.experts(counts, self._scale)
        partial = torch.zeros(n, h, dtype=torch.float32, device=self.device)
        if p:
            partial.index_add_(0, r, y[:p].float())
        out, _ = self.op.combine(partial)
        return out

    def check(self):
        """Raises if an expert GEMM reported an error (synchronises)."""
        self.experts.check()


__all__ = ["CollectiveEpOp", "CollectiveMoE"]
