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
3. receive: per-expert counts, the expert-major row assignment and the
   dequantised bf16 expert-major rows;
4. experts: tcgen05 grouped GEMM (SwiGLU fused) over the expert-major rows
   (TMA-fed; ``native.gather_a = True`` instead gathers and dequantises the A
   tiles straight from the receive slots in producer warps, which skips the
   copy but measured slower), then grouped GEMM whose
   epilogue multiplies by the routing weight and stores every row straight
   into its token owner's top-k slot over NVLink (fused combine; the last CTA
   signals every rank), bf16 compute with fp32 accumulation;
5. combine: each token's top-k rows summed (fp32) into the output.
   ``native.fused_combine = False`` selects the unfused path instead: GEMM2 to
   local memory, per-slot sums sent over NVLink, reduced per token.

``stage(...)`` methods expose the phases separately for profiling,
``set_debug_timing_enabled`` / ``get_debug_timing_snapshot`` record every
kernel's device span per round (:func:`debug_phases` turns a snapshot into a
per-phase table), and
:class:`EpDispatchCombine` gives the reference's transport-only
dispatch/combine contract (rows in, rows out).
"""
import os

import torch

from .._native import load as _load
from ..models import moe as moe_model
from ..utils import dist as kdist
from .p2p import SymmetricHeap

_C = _load()

QUANTS = ("fp8", "nvfp4", "none")

_NVTX = os.environ.get("KIWI_NVTX", "0") not in ("", "0")


class _nvtx_range:
    """An NVTX range around a host call when KIWI_NVTX=1 (no-op otherwise)."""

    __slots__ = ("name",)

    def __init__(self, name):
        self.name = name

    def __enter__(self):
        if _NVTX:
            torch.cuda.nvtx.range_push(self.name)

    def __exit__(self, *exc):
        if _NVTX:
            torch.cuda.nvtx.range_pop()
        return False


def debug_phases(snapshot):
    """Per-kernel device spans of a debug-timing snapshot.

    Returns ``{phase: {"start_us", "end_us", "us"[, "wait_start_us", "wait_end_us", "wait_us"]}}``
    in microseconds relative to the round's earliest stamp, for the phases that
    ran in the round.  ``start`` is the first block's start and ``end`` the last
    warp's exit over the whole grid; the wait entries are block 0's flag wait
    in the receive-side kernels (from its first poll until every source rank's
    flag was seen).  Phase
    words follow the native layout: four per phase, {start, end, wait start,
    wait end}, absolute %globaltimer nanoseconds, 0 = not recorded.
    """
    ticks = list(snapshot["time_ticks"])
    names = list(snapshot["phase_names"])
    t0 = min((t for t in ticks if t), default=0)
    out = {}
    for p, name in enumerate(names):
        w = ticks[4 * p:4 * p + 4]
        if len(w) < 4 or not w[0] or not w[1]:
            continue
        d = {"start_us": (w[0] - t0) / 1e3, "end_us": (w[1] - t0) / 1e3, "us": (w[1] - w[0]) / 1e3}
        if w[2] and w[3]:
            d.update(wait_start_us=(w[2] - t0) / 1e3, wait_end_us=(w[3] - t0) / 1e3, wait_us=(w[3] - w[2]) / 1e3)
        out[name] = d
    return out


def format_debug_timing(snapshot, label="ep"):
    """Human-readable lines of :func:`debug_phases` (one per phase, in start order)."""
    meta = dict(zip(snapshot.get("meta_names", []), snapshot.get("meta", [])))
    head = f"# {label} debug timing rank={meta.get('rank', '?')} world={meta.get('world', '?')} " \
           f"tokens={meta.get('tokens', '?')} recv_tokens={meta.get('recv_tokens', '?')} " \
           f"expert_rows={meta.get('expert_rows', '?')}"
    lines = [head]
    phases = sorted(debug_phases(snapshot).items(), key=lambda kv: kv[1]["start_us"])
    for name, d in phases:
        wait = f" wait={d['wait_us']:.2f}us" if "wait_us" in d else ""
        lines.append(f"#   {name:<13} start={d['start_us']:9.2f}us end={d['end_us']:9.2f}us dur={d['us']:8.2f}us{wait}")
    return "\n".join(lines)


class _DebugTimingMixin:
    """set_debug_timing_enabled / get_debug_timing_snapshot of the reference's
    KiwiEpOp (apps/ep/python/kiwi_ep_bindings.hip.cpp:471-506 of AMDResearch/kiwi),
    backed by the native op's per-kernel %globaltimer spans."""

    def _debug_native(self):
        raise NotImplementedError

    def set_debug_timing_enabled(self, enabled=True):
        self._debug_native().set_debug_timing_enabled(bool(enabled))

    @property
    def debug_timing_enabled(self):
        return self._debug_native().debug_timing_enabled

    def get_debug_timing_snapshot(self):
        """Synchronises the current stream; refused while a CUDA graph is being captured."""
        snap = self._debug_native().get_debug_timing_snapshot()
        snap["phases"] = debug_phases(snap)
        return snap


def layer_config(cfg, rank, world, max_tokens=None):
    """The native EpConfig (dict) of a MoEConfig on `world` ranks."""
    d = dict(world=world, rank=rank, hidden=cfg.hidden, num_experts=cfg.num_experts, topk=cfg.topk,
             max_tokens=max_tokens or cfg.tokens_per_rank, quant=cfg.quant)
    return _C.ep.finalize_config(d)


class ExpertParallelMoE(_DebugTimingMixin):
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
        with _nvtx_range("kiwi.ep.forward"):
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

    def _debug_native(self):
        return self._layer


class EpDispatchCombine(_DebugTimingMixin):
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
        # The caller supplies expert outputs as rows: combine sends them with the
        # combine-send kernel, not through the fused GEMM2 epilogue.
        self.moe.native.fused_combine = False
        # dispatch() returns the expert-major bf16 rows, so the receive side
        # must materialise them (GEMM1's in-place gather skips that copy).
        self.moe.native.gather_a = False
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

    def _debug_native(self):
        return self.moe.native


def _to_send_flat_idx(pos, max_tokens, world):
    """Receive-slot positions (src_rank * max_tokens + token, as the receive
    kernels record them) -> src_rank * (world * max_tokens) + token."""
    return (pos // max_tokens) * (world * max_tokens) + pos % max_tokens


class KiwiEpOp(_DebugTimingMixin):
    """Expert-parallel dispatch/combine with the reference's operator contract
    (``KiwiEpOp`` of apps/ep/python/kiwi_ep_bindings.hip.cpp:123-574 of
    AMDResearch/kiwi, MORI ``EpDispatchCombineOp`` compatible):

    * ``dispatch(input, weights, scales, indices)`` -> ``(out, out_weights,
      out_scales, out_indices, recv_count)``: the rows this rank received, one
      per (source rank, token) that routes at least one expert here, in
      (source rank, token) order, as operator-owned views.  ``out`` holds the
      wire format (``dispatch_dtype`` bf16, or FP8 e4m3 bytes with fp32 1x128
      scales in ``out_scales``, or packed NVFP4 with e4m3 block scales after a
      4-byte fp32 row scale).  The quantisation happens inside dispatch, so
      ``scales`` is accepted and ignored.
    * ``combine(input, weights, indices, out=None)`` -> ``(out, None)``: row i
      of ``input`` goes back to the rank and token it came from; each token's
      rows are summed (no routing weights applied, as MORI).
    """

    _DTYPES = {torch.bfloat16: "none", torch.float8_e4m3fn: "fp8", "fp8": "fp8", "nvfp4": "nvfp4", "none": "none"}

    _QUANT_FORMATS = {"none": None, "fp8": "fp8", "fp4": "nvfp4"}

    def __init__(self, device_id=None, world_size=None, hidden_dim=None, topk=None, num_experts_per_rank=None,
                 max_num_inp_token_per_rank=None, dispatch_dtype=torch.bfloat16, combine_dtype=torch.bfloat16,
                 *_launch_args, group=None, timeout_s=5.0, dispatch_quant_format="none", combine_quant_format="none",
                 **_ignored):
        """Arguments in the reference's order and names (device_id, world_size,
        hidden_dim, topk, num_experts_per_rank, max_num_inp_token_per_rank,
        dispatch_dtype, combine_dtype, ...); its launch arguments (num_blocks,
        num_proxy_threads, scale sizes, queue_capacity, rcomp_backend, ...) are
        accepted and ignored.  ``device_id`` selects the CUDA device and
        ``world_size`` must equal the size of ``group``.  The wire format is
        ``dispatch_quant_format`` ("fp8" / "fp4") when given, else follows
        ``dispatch_dtype``; dispatch always takes bf16 rows and quantises them."""
        missing = [n for n, v in (("hidden_dim", hidden_dim), ("topk", topk),
                                  ("num_experts_per_rank", num_experts_per_rank),
                                  ("max_num_inp_token_per_rank", max_num_inp_token_per_rank)) if v is None]
        if missing:
            raise TypeError("KiwiEpOp missing required arguments: " + ", ".join(missing))
        if combine_dtype != torch.bfloat16 or str(combine_quant_format).lower() != "none":
            raise ValueError("combine_dtype must be torch.bfloat16 (combine_quant_format 'none')")
        fmt = str(dispatch_quant_format).lower()
        if fmt not in self._QUANT_FORMATS:
            raise ValueError(f"unsupported dispatch_quant_format {dispatch_quant_format!r} (none, fp8 or fp4)")
        quant = self._QUANT_FORMATS[fmt] or self._DTYPES.get(dispatch_dtype)
        if quant is None:
            raise ValueError(f"unsupported dispatch_dtype {dispatch_dtype}")
        if device_id is not None:
            torch.cuda.set_device(int(device_id))
        self.group = group
        self.rank = kdist.rank(group)
        self.world_size = kdist.world_size(group)
        if world_size is not None and int(world_size) != self.world_size:
            raise ValueError(f"world_size {world_size} differs from the process group's {self.world_size}")
        self.hidden_dim = hidden_dim
        self.topk = topk
        self.max_tokens = max_num_inp_token_per_rank
        self.layout = _C.ep.finalize_config(dict(
            world=self.world_size, rank=self.rank, hidden=hidden_dim, num_experts=num_experts_per_rank * self.world_size,
            topk=topk, max_tokens=max_num_inp_token_per_rank, quant=quant))
        self.heap = SymmetricHeap(self.layout["heap_bytes"], group)
        self._op = _C.ep.Transport(self.heap.native, self.layout, int(timeout_s * 1e9))
        self._quant = quant
        self._last_tokens = 0
        self._out = None

    def dispatch(self, input, weights, scales=None, indices=None, **_launch_kwargs):
        rows, w, sc, idx, count = self._op.dispatch(input.contiguous(), indices.to(torch.int32).contiguous(),
                                                    weights.float().contiguous())
        self._last_tokens = input.shape[0]
        self._count = count
        if self._quant == "none":
            rows = rows.view(torch.bfloat16)
        elif self._quant == "fp8":
            rows = rows.view(torch.float8_e4m3fn)
            sc = sc.view(torch.float32)
        return rows, w, (None if self._quant == "none" else sc), idx, count

    dispatch_send = dispatch

    def dispatch_recv(self, **_kwargs):
        """dispatch() already completes the receive (kept for call-shape parity)."""

    def combine(self, input, weights=None, indices=None, out=None, **_launch_kwargs):
        t = self._last_tokens
        if out is None:
            if self._out is None or self._out.shape[0] < self.max_tokens:
                self._out = torch.empty(self.max_tokens, self.hidden_dim, dtype=torch.bfloat16, device=input.device)
            out = self._out[:t]
        self._op.combine(input.contiguous(), out)
        return out, None

    combine_send = combine

    def combine_recv(self, **_kwargs):
        return self._out[:self._last_tokens] if self._out is not None else None, None

    def reset(self):
        """Ends the current round on the host.  Device slots are epoch-tagged,
        so nothing on the GPU needs clearing; like the reference, the call is
        refused while the current stream is being captured into a graph and
        otherwise waits for the stream."""
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("KiwiEpOp.reset() is not supported during graph capture; dispatch and combine "
                               "already carry their per-round state on the device")
        torch.cuda.current_stream().synchronize()
        self._last_tokens = 0

    def max_num_tokens_to_recv(self):
        return self.world_size * self.max_tokens

    def max_num_tokens_to_recv_per_rank(self):
        return self.max_tokens

    def max_num_tokens_to_send(self):
        return self.world_size * self.max_tokens

    def max_num_tokens_to_send_per_rank(self):
        return self.max_tokens

    def launch_policy(self, num_tokens):
        """The launch configuration dispatch / combine use (the B200 tuning
        table with KIWI_EP_TUNING applied): grid sizes of the EP kernels, the
        transport and the table's source.  ``num_tokens`` is accepted for call
        compatibility; the table is keyed by the op's configuration."""
        sms = _default_sms()
        t = dict(_C.ep.tune(self.layout, sms, os.environ.get("KIWI_EP_TUNING")))
        t.update(num_tokens=int(num_tokens), num_blocks=_C.ep.dispatch_grid(int(num_tokens), 0, sms),
                 transport="nvlink", gpu_arch="sm_100a")
        return t

    def decode_send_flat_idx(self, flat_idx):
        """(source rank, source token) of a position from get_dispatch_src_token_pos()."""
        stride = self.max_num_tokens_to_send()
        return int(flat_idx) // stride, int(flat_idx) % stride

    def get_dispatch_src_token_pos(self):
        """Source position of each row received by the last dispatch, encoded as
        ``src_rank * max_num_tokens_to_send() + src_token`` (the reference's
        encoding; decode_send_flat_idx inverts it).  Reads the received count,
        so it synchronises the current stream."""
        n = int(self._count.item()) if getattr(self, "_count", None) is not None else 0
        return _to_send_flat_idx(self._op.src_token_pos[:n], self.max_tokens, self.world_size)

    def get_registered_combine_input_buffer(self, combine_dtype=torch.bfloat16, hidden_dim=-1):
        """Operator-owned [max_num_tokens_to_recv(), hidden] buffer a caller can
        write expert outputs into and pass to combine() without a copy."""
        if combine_dtype != torch.bfloat16:
            raise ValueError("combine_dtype must be torch.bfloat16")
        if hidden_dim > 0 and hidden_dim != self.hidden_dim:
            raise ValueError("get_registered_combine_input_buffer hidden_dim must match the configured hidden_dim")
        buf = getattr(self, "_combine_in", None)
        if buf is None:
            dev = torch.device("cuda", torch.cuda.current_device())
            buf = self._combine_in = torch.empty(self.max_num_tokens_to_recv(), self.hidden_dim,
                                                 dtype=torch.bfloat16, device=dev)
        return buf

    def _debug_native(self):
        return self._op

    def check(self):
        code, site, info, rank = self._op.error()
        if code:
            raise RuntimeError(f"kiwi ep error: code={code} site={site} info={info} rank={rank}")


# ---- module-level helpers of the reference's extension (kiwi_ep_ext) ----

def barrier(group=None):
    """Host barrier over the process group (the reference's LCI barrier)."""
    kdist.barrier(group)


def get_rank(group=None):
    """This process's rank in `group`."""
    return kdist.rank(group)


def get_nranks(group=None):
    """Number of ranks in `group`."""
    return kdist.world_size(group)


def get_hca_name_for_gpu(device=None):
    """Always "": every peer is reached over NVLink, no NIC is selected."""
    return ""


def get_hca_name_for_current_gpu():
    """Always "": every peer is reached over NVLink."""
    return ""


def _default_sms():
    try:
        if torch.cuda.is_available():
            return torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    except Exception:  # noqa: BLE001
        pass
    return 148  # B200


def recommended_runtime_defaults(num_tokens, world_size, gpu_arch="", nic_family="", hidden_dim=7168,
                                 num_experts=256, topk=8, quant="fp8"):
    """Launch defaults the B200 tuning table gives an op of `num_tokens` tokens
    per rank on `world_size` ranks (KIWI_EP_TUNING applied).  gpu_arch and
    nic_family are accepted for call compatibility: the table is keyed by the
    configuration and this GPU's SM count."""
    cfg = dict(world=int(world_size), rank=0, hidden=hidden_dim, num_experts=num_experts, topk=topk,
               max_tokens=max(1, int(num_tokens)), quant=quant)
    sms = _default_sms()
    t = dict(_C.ep.tune(cfg, sms, os.environ.get("KIWI_EP_TUNING")))
    t.update(num_blocks=_C.ep.dispatch_grid(int(num_tokens), t["dispatch_blocks"], sms), rcomp_backend="nvlink")
    return t


def recommended_num_blocks(num_tokens, world_size, gpu_arch="", nic_family=""):
    """Dispatch grid size of recommended_runtime_defaults."""
    return recommended_runtime_defaults(num_tokens, world_size, gpu_arch, nic_family)["num_blocks"]


__all__ = ["ExpertParallelMoE", "EpDispatchCombine", "KiwiEpOp", "layer_config", "debug_phases",
           "format_debug_timing", "barrier", "get_rank", "get_nranks", "get_hca_name_for_gpu",
           "get_hca_name_for_current_gpu", "recommended_num_blocks", "recommended_runtime_defaults"]
