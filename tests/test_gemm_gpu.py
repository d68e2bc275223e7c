"""tcgen05 grouped BF16 GEMM vs a plain PyTorch fp32 reference of the same op."""
import pytest
import torch

import kiwi_b200

pytestmark = pytest.mark.gpu


def _ref(a, b, counts, n, swiglu, row_scale=None):
    outs = []
    off = 0
    for g, c in enumerate(counts):
        ag = a[off:off + c].float()
        bg = b[g * n:(g + 1) * n].float()
        y = ag @ bg.t()
        if swiglu:
            cols = []
            for t in range(n // 256):
                gate = y[:, t * 256:t * 256 + 128]
                up = y[:, t * 256 + 128:t * 256 + 256]
                cols.append(torch.nn.functional.silu(gate) * up)
            y = torch.cat(cols, dim=1)
        if row_scale is not None:
            y = y * row_scale[off:off + c, None]
        outs.append(y)
        off += c
    return torch.cat(outs, 0)


@pytest.mark.parametrize("pair", [False, True])
@pytest.mark.parametrize("counts,n,k,swiglu", [
    ([5, 130, 0, 256], 256, 128, False),
    ([128], 512, 64, False),
    ([1, 0, 300], 512, 192, True),
    ([257, 64], 1024, 7168 // 4, True),
])
def test_grouped_gemm_matches_fp32(counts, n, k, swiglu, pair):
    torch.manual_seed(0)
    C = kiwi_b200.native()
    rows = sum(counts)
    a = (torch.randn(max(rows, 1), k, device="cuda") * 0.5).bfloat16()
    b = (torch.randn(len(counts) * n, k, device="cuda") * 0.05).bfloat16()
    out = torch.full((max(rows, 1), n // 2 if swiglu else n), float("nan"), device="cuda", dtype=torch.bfloat16)
    plan = C.ops.GroupedGemm(a, b, len(counts))
    cnt = torch.tensor(counts, dtype=torch.int32, device="cuda")
    scale = torch.rand(max(rows, 1), device="cuda") + 0.5
    plan.run(cnt, out, swiglu, scale, 0, pair)
    torch.cuda.synchronize()
    assert int(plan.error.item()) == 0
    ref = _ref(a, b, counts, n, swiglu, scale)
    got = out[:rows].float()
    assert torch.isfinite(got).all()
    err = (got - ref).abs().max().item()
    tol = 2e-2 * ref.abs().max().item() + 1e-2
    assert err <= tol, (err, tol)


@pytest.mark.parametrize("swiglu", [False, True])
def test_bk32_stages_match_bk64_bitwise(swiglu):
    """The opt-in 32-column-stage kernel (64-byte swizzle, 9 stages) issues the
    same K = 16 MMAs in the same order as the default 64-column one, so the
    outputs are identical, ragged and empty groups included."""
    torch.manual_seed(1)
    C = kiwi_b200.native()
    counts, n, k = [200, 0, 256, 77], 512, 1024
    rows = sum(counts)
    a = (torch.randn(rows, k, device="cuda") * 0.5).bfloat16()
    b = (torch.randn(len(counts) * n, k, device="cuda") * 0.05).bfloat16()
    cols = n // 2 if swiglu else n
    o64 = torch.full((rows, cols), float("nan"), device="cuda", dtype=torch.bfloat16)
    o32 = torch.full_like(o64, float("nan"))
    plan = C.ops.GroupedGemm(a, b, len(counts))
    cnt = torch.tensor(counts, dtype=torch.int32, device="cuda")
    plan.run(cnt, o64, swiglu)
    plan.run(cnt, o32, swiglu, None, 0, False, None, 32)
    torch.cuda.synchronize()
    assert int(plan.error.item()) == 0
    assert torch.isfinite(o64.float()).all()
    assert torch.equal(o64, o32)


@pytest.mark.parametrize("bk", [64, 32])
@pytest.mark.parametrize("swiglu", [False, True])
def test_m64_tail_tiles_match_m128_bitwise(swiglu, bk):
    """Tiles with at most 64 rows of their group left run M = 64 MMAs (the
    default) and give the same bits as M = 128 MMAs over the same K order, and
    the fp32 reference within tolerance.  Groups leave tails of 1, 5, 6, 44,
    64 and 65 rows, plus empty and whole-tile groups."""
    torch.manual_seed(5)
    C = kiwi_b200.native()
    counts = [70, 0, 200, 5, 64, 65, 1, 128, 130, 300]
    k, n = 512, 512
    rows, groups = sum(counts), len(counts)
    a = (torch.randn(rows, k, device="cuda") * 0.5).bfloat16()
    b = (torch.randn(groups * n, k, device="cuda") * 0.05).bfloat16()
    cnt = torch.tensor(counts, dtype=torch.int32, device="cuda")
    scale = torch.rand(rows, device="cuda") + 0.5
    cols = n // 2 if swiglu else n
    plan = C.ops.GroupedGemm(a, b, groups)
    m128 = torch.zeros(rows, cols, device="cuda", dtype=torch.bfloat16)
    plan.run(cnt, m128, swiglu, scale, 0, False, None, bk, False)
    m64 = torch.full((rows, cols), 3.0, device="cuda", dtype=torch.bfloat16)
    plan.run(cnt, m64, swiglu, scale, 0, False, None, bk, True)
    torch.cuda.synchronize()
    assert int(plan.error.item()) == 0
    assert torch.equal(m64, m128)
    exact = _ref(a, b, counts, n, swiglu, scale)
    assert (m64.float() - exact).abs().max().item() <= 2e-2 * exact.abs().max().item() + 1e-2


@pytest.mark.parametrize("pair", [False, True])
@pytest.mark.parametrize("swiglu", [False, True])
def test_blocked_weights_match_row_major_bitwise(swiglu, pair):
    """B in the blocked layout (one contiguous 256 x 64 box per TMA load) gives
    the same bits as row-major B, on the 1-SM and the 2-SM kernel."""
    from kiwi_b200.ops import block_weights

    torch.manual_seed(6)
    C = kiwi_b200.native()
    counts = [300, 0, 129, 64, 512]
    k, n = 448, 768
    rows, groups = sum(counts), len(counts)
    a = (torch.randn(rows, k, device="cuda") * 0.5).bfloat16()
    b = (torch.randn(groups * n, k, device="cuda") * 0.05).bfloat16()
    cnt = torch.tensor(counts, dtype=torch.int32, device="cuda")
    cols = n // 2 if swiglu else n
    ref = torch.zeros(rows, cols, device="cuda", dtype=torch.bfloat16)
    C.ops.GroupedGemm(a, b, groups).run(cnt, ref, swiglu, None, 0, pair)
    plan = C.ops.GroupedGemm(a, block_weights(b, groups), groups, b_blocked=True)
    got = torch.full((rows, cols), 5.0, device="cuda", dtype=torch.bfloat16)
    plan.run(cnt, got, swiglu, None, 0, pair)
    torch.cuda.synchronize()
    assert int(plan.error.item()) == 0
    assert torch.equal(got, ref)
    exact = _ref(a, b, counts, n, swiglu)
    assert (got.float() - exact).abs().max().item() <= 2e-2 * exact.abs().max().item() + 1e-2


def test_gemm_kernels_use_no_local_memory():
    C = kiwi_b200.native()
    for sw in (False, True):
        local, regs, smem = C.ops.gemm_kernel_info(sw)
        assert local == 0, (sw, local)
        local, regs, smem = C.ops.gemm_pair_kernel_info(sw)
        assert local == 0, (sw, local)
    for pair in (False, True):
        local, regs, smem = C.ops.gemm_scatter_kernel_info(pair)
        assert local == 0 and smem <= 227 * 1024, (pair, local, smem)


@pytest.mark.parametrize("pair", [False, True])
def test_grouped_gemm_large_rows(pair):
    """Groups with several 256-row tiles and ragged tails (both kernels)."""
    torch.manual_seed(3)
    C = kiwi_b200.native()
    counts = [700, 256, 1, 513]
    n, k = 512, 256
    rows = sum(counts)
    a = (torch.randn(rows, k, device="cuda") * 0.5).bfloat16()
    b = (torch.randn(len(counts) * n, k, device="cuda") * 0.05).bfloat16()
    out = torch.zeros(rows, n, device="cuda", dtype=torch.bfloat16)
    C.ops.GroupedGemm(a, b, len(counts)).run(torch.tensor(counts, dtype=torch.int32, device="cuda"), out, False,
                                             None, 0, pair)
    torch.cuda.synchronize()
    ref = _ref(a, b, counts, n, False)
    assert (out.float() - ref).abs().max().item() <= 2e-2 * ref.abs().max().item() + 1e-2


@pytest.mark.parametrize("swiglu", [False, True])
def test_ops_plan_runs_the_kernel_and_matches_its_reference(swiglu):
    """kiwi_b200.ops.GroupedGemm on CUDA tensors (the tcgen05 kernel) against
    kiwi_b200.ops.grouped_gemm_reference, the fp32 path CPU tensors take."""
    from kiwi_b200.ops import GroupedGemm, grouped_gemm_reference

    torch.manual_seed(5)
    counts, n, k = [64, 0, 130], 512, 256
    rows = sum(counts)
    a = (torch.randn(rows, k, device="cuda") * 0.5).bfloat16()
    b = (torch.randn(len(counts) * n, k, device="cuda") * 0.05).bfloat16()
    scale = torch.rand(rows, device="cuda") + 0.5
    plan = GroupedGemm(a, b, len(counts))
    assert plan._plan is not None  # the native kernel, not the reference
    out = plan(counts, swiglu=swiglu, row_scale=scale)
    torch.cuda.synchronize()
    plan.check()
    ref = grouped_gemm_reference(a, b, counts, swiglu, scale)
    assert (out[:rows].float() - ref).abs().max().item() <= 2e-2 * ref.abs().max().item() + 1e-2


@pytest.mark.parametrize("experts,topk", [(8, 2), (64, 6), (256, 8)])
def test_ops_route_topk_matches_the_reference(experts, topk):
    """kiwi_b200.ops.route_topk (the EP layer's routing kernel) against
    torch.topk + softmax in fp32."""
    from kiwi_b200.models import moe
    from kiwi_b200.ops import route_topk

    torch.manual_seed(experts)
    logits = torch.randn(300, experts, device="cuda")
    idx, w = route_topk(logits, topk)
    ridx, rw = moe.route_reference(logits, topk)
    assert torch.equal(idx, ridx)
    assert torch.allclose(w, rw, atol=1e-6)


def test_expert_ffn_blocked_weights_match_rows_and_reference():
    """kiwi_b200.ops.ExpertFFN with its default blocked weight copies gives the
    row-major op's bits, and the MoE reference's expert math within tolerance."""
    from kiwi_b200.ops import ExpertFFN, grouped_gemm_reference

    torch.manual_seed(7)
    e, hidden, ffn, counts = 4, 512, 256, [70, 0, 200, 33]
    rows = sum(counts)
    w13 = (torch.randn(e * 2 * ffn, hidden, device="cuda") * 0.05).bfloat16()
    w2 = (torch.randn(e * hidden, ffn, device="cuda") * 0.05).bfloat16()
    x = (torch.randn(rows, hidden, device="cuda") * 0.5).bfloat16()
    scale = torch.rand(rows, device="cuda") + 0.5
    outs = {}
    for layout in ("blocked", "rows"):
        op = ExpertFFN(w13, w2, e, rows, weight_layout=layout)
        assert op.gemm1.b_layout == layout
        op.input_buffer()[:rows].copy_(x)
        outs[layout] = op(counts, scale)[:rows].clone()
        op.check()
    assert torch.equal(outs["blocked"], outs["rows"])
    h = grouped_gemm_reference(x, w13, counts, swiglu=True).bfloat16()
    ref = grouped_gemm_reference(h, w2, counts, row_scale=scale)
    assert (outs["blocked"].float() - ref).abs().max().item() <= 3e-2 * ref.abs().max().item() + 1e-2
