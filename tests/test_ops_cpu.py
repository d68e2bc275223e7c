"""kiwi_b200.ops on CPU tensors: the grouped GEMM's fp32 restatement against a
plain per-group matmul, and the expert FFN against the MoE reference's math."""
import pytest
import torch
import torch.nn.functional as F

from kiwi_b200.models import moe
from kiwi_b200.ops import ExpertFFN, GroupedGemm, grouped_gemm, grouped_gemm_reference


def _plain(a, b, counts, swiglu, row_scale):
    n = b.shape[0] // len(counts)
    outs, off = [], 0
    for g, c in enumerate(counts):
        y = a[off:off + c].double() @ b[g * n:(g + 1) * n].double().t()
        if swiglu:
            y = torch.cat([F.silu(y[:, t:t + 128]) * y[:, t + 128:t + 256] for t in range(0, n, 256)], 1)
        if row_scale is not None:
            y = y * row_scale[off:off + c].double()[:, None]
        outs.append(y)
        off += c
    return torch.cat(outs)


@pytest.mark.parametrize("swiglu", [False, True])
@pytest.mark.parametrize("counts", [[5, 0, 17], [0, 0], [33]])
def test_reference_matches_per_group_matmul(counts, swiglu):
    torch.manual_seed(0)
    rows, k, n = sum(counts), 64, 512
    a = torch.randn(max(rows, 1), k).bfloat16()
    b = (torch.randn(len(counts) * n, k) * 0.1).bfloat16()
    scale = torch.rand(max(rows, 1)) + 0.5
    got = grouped_gemm_reference(a, b, counts, swiglu, scale)
    assert got.shape == (rows, n // 2 if swiglu else n)
    if rows:
        assert torch.allclose(got.double(), _plain(a, b, counts, swiglu, scale), rtol=1e-5, atol=1e-5)


def test_plan_on_cpu_tensors_writes_only_the_counted_rows():
    torch.manual_seed(1)
    a = torch.randn(12, 64).bfloat16()
    b = (torch.randn(2 * 256, 64) * 0.1).bfloat16()
    out = torch.full((12, 256), 7.0).bfloat16()
    GroupedGemm(a, b, 2)([3, 4], out)
    ref = grouped_gemm_reference(a[:7], b, [3, 4]).bfloat16()
    assert torch.equal(out[:7], ref) and (out[7:] == 7).all()
    one = grouped_gemm(a, b, torch.tensor([3, 4]))
    assert torch.equal(one[:7], ref)
    with pytest.raises(ValueError):
        GroupedGemm(a, b[:-1], 2)


def test_expert_ffn_matches_the_moe_reference():
    cfg = moe.MoEConfig(hidden=256, ffn=128, num_experts=3, topk=1, tokens_per_rank=8, quant="none", name="t")
    w13, w2 = moe.local_expert_weights(cfg, 0, 1, "cpu")
    ffn = ExpertFFN(w13, w2, 3, 16)
    torch.manual_seed(2)
    x = torch.randn(10, 256).bfloat16()
    counts = [4, 0, 6]
    scale = torch.rand(16)
    ffn.input_buffer()[:10].copy_(x)
    y = ffn(torch.tensor(counts), scale)[:10].float()
    off = 0
    for e, c in enumerate(counts):
        if c == 0:
            continue
        g, u, d = moe.expert_weights(cfg, e, "cpu")
        a = x[off:off + c].float()
        hid = (F.silu(a @ g.float().t()) * (a @ u.float().t())).bfloat16().float()
        want = (hid @ d.float().t()) * scale[off:off + c, None]
        assert (y[off:off + c] - want).abs().max().item() <= 1e-2 * want.abs().max().item() + 1e-4
        off += c
    with pytest.raises(ValueError):
        ExpertFFN(w13, w2[:-1], 3, 4)


def test_row_copies_on_cpu_follow_the_index_rules():
    from kiwi_b200.ops import accumulate_rows, check_error, copy_rows

    src = torch.arange(5 * 8, dtype=torch.float32).view(5, 8).bfloat16()
    dst = torch.zeros(4, 8).bfloat16()
    err = copy_rows(src, dst, torch.tensor([4, -1, 9, 0]), torch.tensor([0, 1, 2, 7]))
    assert err == 1 | 2  # index 9 past src, 7 past dst: both rows skipped
    assert torch.equal(dst[0], src[4]) and (dst[1:] == 0).all()
    with pytest.raises(RuntimeError):
        check_error(err)
    check_error(0)
    out, err = accumulate_rows(src, torch.tensor([[0, 1], [-1, -1], [2, 7]]))
    assert err == 1 and torch.equal(out[0], (src[0].float() + src[1].float()).bfloat16())
    assert (out[1] == 0).all() and torch.equal(out[2], src[2])


def test_ep_copy_bench_accounting():
    import importlib.util
    import pathlib

    path = pathlib.Path(__file__).resolve().parent.parent / "benchmarks" / "bench_ep_copy.py"
    spec = importlib.util.spec_from_file_location("bench_ep_copy", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    assert mod.algorithmic_bytes("copy", 16384, 7168, 8) == 2 * 16384 * 7168 * 2
    assert mod.algorithmic_bytes("accumulate", 16384, 7168, 8) == (16384 + 2048) * 7168 * 2
    src, dst, idx = mod.build("accumulate", 64, 16, 8, "cpu")
    assert tuple(idx.shape) == (8, 8) and sorted(idx.view(-1).tolist()) == list(range(64))
    src, dst, idx = mod.build("copy", 64, 16, 8, "cpu")
    assert idx is None and dst.shape == src.shape
    peak, how = mod.hbm_peak("/nonexistent/peaks.json")
    assert (peak, how) == (mod.FALLBACK_HBM_GBS, "fallback")
    assert mod.agree("accumulate", torch.ones(2, 2), torch.ones(2, 2) * 1.001)
    assert not mod.agree("pack", torch.ones(2, 2), torch.ones(2, 2) * 1.001)


def test_route_topk_on_cpu_is_the_reference():
    from kiwi_b200.ops import route_topk

    logits = torch.randn(9, 16)
    idx, w = route_topk(logits, 4)
    ridx, rw = moe.route_reference(logits, 4)
    assert torch.equal(idx, ridx) and torch.equal(w, rw)
    assert idx.dtype == torch.int32 and torch.allclose(w.sum(-1), torch.ones(9))


def test_quant_fp8_on_cpu_is_the_reference():
    from kiwi_b200.ops import quant_fp8

    x = torch.randn(4, 256).bfloat16()
    codes, scales = quant_fp8(x)
    rc, rs = moe.quant_fp8_codes(x)
    assert torch.equal(codes.view(torch.uint8), rc.view(torch.uint8)) and torch.equal(scales, rs)


def test_block_weights_places_each_box_contiguously_and_round_trips():
    """block_weights: the 256 x 64 box of (group g, n-tile nt, k-block kb) is
    rows [r, r + 256) of the [G * N * K / 64, 64] result with
    r = ((g * N / 256 + nt) * K / 64 + kb) * 256; unblock_weights inverts it."""
    from kiwi_b200.ops import block_weights, unblock_weights

    g, n, k = 3, 512, 192
    w = torch.randn(g * n, k).to(torch.bfloat16)
    wb = block_weights(w, g)
    assert wb.shape == (g * n * k // 64, 64) and wb.is_contiguous()
    for gi, nt, kb in [(0, 0, 0), (1, 1, 2), (2, 0, 1), (2, 1, 2)]:
        r = ((gi * (n // 256) + nt) * (k // 64) + kb) * 256
        box = w[gi * n + nt * 256:gi * n + nt * 256 + 256, kb * 64:kb * 64 + 64]
        assert torch.equal(wb[r:r + 256], box)
    assert torch.equal(unblock_weights(wb, g, k), w)
    with pytest.raises(ValueError):
        block_weights(torch.zeros(3 * 100, 64), 3)


def test_blocked_layout_request_on_cpu_keeps_row_major_reference():
    """b_layout="blocked" only changes what the CUDA kernel reads; CPU tensors
    keep the row-major B and the fp32 reference path, and a bad layout name
    raises."""
    torch.manual_seed(1)
    a = torch.randn(40, 128).bfloat16()
    b = (torch.randn(2 * 256, 128) * 0.05).bfloat16()
    plan = GroupedGemm(a, b, 2, b_layout="blocked")
    assert plan.b_layout == "rows" and plan.b is b
    out = plan([30, 10])
    assert torch.allclose(out[:40].float(), grouped_gemm_reference(a, b, [30, 10]), atol=1e-2)
    with pytest.raises(ValueError):
        GroupedGemm(a, b, 2, b_layout="tiled")
    ffn = ExpertFFN(torch.zeros(2 * 2 * 128, 128).bfloat16(), torch.zeros(2 * 128, 128).bfloat16(), 2, 8)
    assert ffn.gemm1.b_layout == "rows"
