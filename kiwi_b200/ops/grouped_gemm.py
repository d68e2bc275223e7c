"""Grouped BF16 GEMM and the expert SwiGLU FFN built from it.

``GroupedGemm(a, b, num_groups)`` computes, for each group g with ``counts[g]``
consecutive rows of ``a`` (``a`` [rows, K] bf16, ``b`` [G * N, K] bf16, group
g's weights in rows g*N .. g*N+N-1):

    out[rows of g] = a[rows of g] @ b[g].T                       (swiglu off)
    out[rows of g] = silu(y_gate) * y_up, per 256-column tile     (swiglu on)

optionally times ``row_scale[row]`` (fp32, one per row).  With SwiGLU the
weights are interleaved in blocks of 128 rows (gate 0..127, up 0..127, gate
128..255, ...; :func:`kiwi_b200.models.moe.interleave_gate_up`), so each
256-column accumulator tile holds a gate block and its up block and the output
has N / 2 columns.

CUDA tensors run the sm_100a tcgen05 kernel (``kiwi_b200._C.ops.GroupedGemm``:
TMA-fed operands, TMEM accumulators, fused SwiGLU / row-scale epilogue; the
extension must be built, nothing falls back).  CPU tensors run
:func:`grouped_gemm_reference`, the fp32 restatement of the same op, so the
layers built on it also run in CPU processes.

Parity: the reference's expert GEMMs are outside its EP library (the caller's
framework runs them; apps/ep/python of AMDResearch/kiwi returns the received
rows); here they are part of the package because the fused EP layer issues
them itself.
"""
import torch
import torch.nn.functional as F

_TILE = 256  # SwiGLU tile: 128 gate columns + 128 up columns


def _swiglu_tiles(y):
    """silu(gate) * up over interleaved 256-column tiles of y [rows, N] -> [rows, N / 2]."""
    rows, n = y.shape
    t = y.view(rows, n // _TILE, 2, _TILE // 2)
    return (F.silu(t[:, :, 0]) * t[:, :, 1]).reshape(rows, n // 2)


def grouped_gemm_reference(a, b, counts, swiglu=False, row_scale=None):
    """fp32 reference of the grouped GEMM (same layout and epilogue as the kernel).

    a [rows, K], b [G * N, K], counts [G] (any integer sequence or tensor);
    returns fp32 [sum(counts), N or N / 2]."""
    counts = [int(c) for c in (counts.tolist() if torch.is_tensor(counts) else counts)]
    g = len(counts)
    n = b.shape[0] // g
    outs, off = [], 0
    for e, c in enumerate(counts):
        y = a[off:off + c].float() @ b[e * n:(e + 1) * n].float().t()
        if swiglu:
            y = _swiglu_tiles(y)
        if row_scale is not None:
            y = y * row_scale[off:off + c].float()[:, None]
        outs.append(y)
        off += c
    if not outs:
        return torch.empty(0, n // 2 if swiglu else n, device=a.device)
    return torch.cat(outs, 0)


def block_weights(w, num_groups):
    """Row-major grouped weights [G * N, K] -> the blocked layout the GEMM
    kernels read with ``b_blocked``: a [G * N * K / 64, 64] matrix in which the
    256-row x 64-column box of group g, n-tile nt and k-block kb is contiguous
    (32 KB) at row ((g * N / 256 + nt) * K / 64 + kb) * 256, so every TMA load
    of a weight tile reads whole DRAM pages.  Returns a new tensor."""
    if w.dim() != 2 or w.shape[0] % num_groups:
        raise ValueError("w must be [num_groups * N, K]")
    n, k = w.shape[0] // num_groups, w.shape[1]
    if n % 256 or k % 64:
        raise ValueError("N must be a multiple of 256 and K of 64")
    return w.view(num_groups, n // 256, 256, k // 64, 64).permute(0, 1, 3, 2, 4).contiguous().view(-1, 64)


def unblock_weights(wb, num_groups, k):
    """Inverse of :func:`block_weights` ([G * N * K / 64, 64] -> [G * N, K])."""
    n = wb.numel() // (num_groups * k)
    return wb.view(num_groups, n // 256, k // 64, 256, 64).permute(0, 1, 3, 2, 4).contiguous().view(-1, k)


class GroupedGemm:
    """A grouped GEMM bound to fixed A and B buffers (the kernel's tensor maps
    are built once; refill ``a`` in place between calls).

    ``__call__(counts, out=None, swiglu=False, row_scale=None, bk=64, pair=False, m64=True)``
    enqueues the GEMM on the current stream and returns ``out`` (bf16, at least
    ``a.shape[0]`` rows; rows past ``sum(counts)`` are left as they were).
    ``bk`` picks the K columns per pipeline stage (64 default; 32 and 128 are
    opt-in 1-SM variants), ``pair`` the 2-SM kernel and ``m64`` M = 64 MMAs on
    1-SM tiles with at most 64 rows of their group left; all compute the same
    result.  :meth:`check` raises if the kernel reported an error (a wait that
    ran out, or a schedule that did not fit ``out``).

    ``b_layout="blocked"`` keeps a copy of ``b`` in the layout of
    :func:`block_weights` for the kernel (each weight load reads one contiguous
    32 KB box; same result) and drops the reference to the row-major ``b`` on
    CUDA (``self.b`` is then the blocked copy); CPU tensors always use ``b`` as
    given."""

    def __init__(self, a, b, num_groups, b_layout="rows"):
        if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[1] or b.shape[0] % num_groups:
            raise ValueError("a [rows, K] and b [num_groups * N, K] are required")
        if b_layout not in ("rows", "blocked"):
            raise ValueError("b_layout must be 'rows' or 'blocked'")
        self.a, self.b, self.num_groups = a, b, int(num_groups)
        self.n, self.k = b.shape[0] // self.num_groups, a.shape[1]
        self.b_layout = b_layout if a.is_cuda else "rows"
        self._plan = None
        if a.is_cuda:
            from .. import native

            if self.b_layout == "blocked":
                self.b = block_weights(b, self.num_groups)
            self._plan = native().ops.GroupedGemm(a, self.b, self.num_groups, b_blocked=self.b_layout == "blocked")

    def out_columns(self, swiglu):
        return self.n // 2 if swiglu else self.n

    def __call__(self, counts, out=None, swiglu=False, row_scale=None, bk=64, pair=False, m64=True):
        cols = self.out_columns(swiglu)
        if out is None:
            out = torch.empty(self.a.shape[0], cols, dtype=torch.bfloat16, device=self.a.device)
        if self._plan is None:
            counts = torch.as_tensor(counts)
            rows = int(counts.sum())
            out[:rows].copy_(grouped_gemm_reference(self.a[:rows], self.b, counts, swiglu,
                                                    None if row_scale is None else row_scale[:rows]))
            return out
        if not torch.is_tensor(counts) or not counts.is_cuda:
            counts = torch.as_tensor(counts, dtype=torch.int32).to(self.a.device)
        self._plan.run(counts.to(torch.int32), out, bool(swiglu), row_scale, 0, bool(pair), None, int(bk), bool(m64))
        return out

    def check(self):
        """Raises RuntimeError if the kernel set its error word (synchronises)."""
        if self._plan is not None:
            err = int(self._plan.error.item())
            if err:
                raise RuntimeError(f"grouped GEMM error word {err:#x}")


def grouped_gemm(a, b, counts, swiglu=False, row_scale=None, out=None, bk=64, pair=False):
    """One-shot :class:`GroupedGemm` (builds the tensor maps on every call; keep a
    GroupedGemm for repeated calls on the same buffers)."""
    g = len(counts) if not torch.is_tensor(counts) else counts.numel()
    return GroupedGemm(a, b, g)(counts, out, swiglu, row_scale, bk, pair)


class ExpertFFN:
    """The SwiGLU FFN of E local experts on expert-sorted rows.

    ``w13`` [E * 2F, H] holds each expert's gate and up weights interleaved in
    128-row blocks, ``w2`` [E * H, F] its down projection.  The op owns an
    input buffer of ``max_rows`` rows (:meth:`input_buffer`); the caller fills
    its first ``sum(counts)`` rows in expert order and calls ``ffn(counts,
    row_scale)``, which runs GEMM1 with the SwiGLU epilogue into the owned
    hidden buffer and GEMM2 with the per-row scale (the routing weight) and
    returns the bf16 rows [max_rows, H] (the first ``sum(counts)`` valid).
    ``weight_layout="blocked"`` (the default) gives both GEMMs blocked copies
    of the weights (:func:`block_weights`; same result, faster weight loads)."""

    def __init__(self, w13, w2, num_experts, max_rows, weight_layout="blocked"):
        e = int(num_experts)
        if w13.shape[0] % (2 * e) or w2.shape[0] % e:
            raise ValueError("w13 must be [E * 2F, H] and w2 [E * H, F]")
        hidden, ffn = w13.shape[1], w13.shape[0] // (2 * e)
        if w2.shape != (e * hidden, ffn):
            raise ValueError(f"w2 must be [{e * hidden}, {ffn}]")
        if ffn % 128:
            raise ValueError("the SwiGLU epilogue needs F to be a multiple of 128")
        dev = w13.device
        self.num_experts, self.hidden, self.ffn, self.max_rows = e, hidden, ffn, int(max_rows)
        rows = max(self.max_rows, 1)
        self._a = torch.zeros(rows, hidden, dtype=torch.bfloat16, device=dev)
        self._h = torch.zeros(rows, ffn, dtype=torch.bfloat16, device=dev)
        self._y = torch.zeros(rows, hidden, dtype=torch.bfloat16, device=dev)
        self.gemm1 = GroupedGemm(self._a, w13, e, b_layout=weight_layout)
        self.gemm2 = GroupedGemm(self._h, w2, e, b_layout=weight_layout)

    def input_buffer(self):
        return self._a

    def __call__(self, counts, row_scale=None):
        self.gemm1(counts, self._h, swiglu=True)
        self.gemm2(counts, self._y, swiglu=False, row_scale=row_scale)
        return self._y

    def check(self):
        self.gemm1.check()
        self.gemm2.check()


__all__ = ["GroupedGemm", "grouped_gemm", "grouped_gemm_reference", "ExpertFFN", "block_weights", "unblock_weights"]
