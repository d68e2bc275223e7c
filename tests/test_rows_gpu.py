"""Row-copy kernels (kiwi_b200.ops.copy_rows / accumulate_rows on CUDA tensors)
against plain PyTorch: gather, scatter, skipped and out-of-range indices, and
the fp32 top-k sum."""
import pytest
import torch

from kiwi_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("hidden", [8, 7168, 7176])
def test_gather_and_scatter_match_torch(hidden):
    torch.manual_seed(0)
    src = torch.randn(300, hidden, device="cuda").bfloat16()
    perm = torch.randperm(300, device="cuda").to(torch.int32)
    dst = torch.zeros_like(src)
    ops.check_error(ops.copy_rows(src, dst, perm))
    assert torch.equal(dst, src[perm.long()])
    dst.zero_()
    ops.check_error(ops.copy_rows(src, dst, None, perm))
    want = torch.zeros_like(src)
    want[perm.long()] = src
    assert torch.equal(dst, want)


def test_skipped_and_out_of_range_rows_are_not_written():
    src = torch.randn(4, 64, device="cuda").bfloat16()
    dst = torch.zeros(4, 64, device="cuda").bfloat16()
    err = ops.copy_rows(src, dst, torch.tensor([3, -1, 4, 1], device="cuda"), torch.tensor([0, 1, 2, 9]))
    assert int(err.item()) == 3  # source index 4 and destination index 9 are past the end
    assert torch.equal(dst[0], src[3]) and (dst[1:] == 0).all()


@pytest.mark.parametrize("k", [1, 3, 8])
def test_accumulate_matches_fp32_sum(k):
    torch.manual_seed(1)
    src = torch.randn(97, 7168, device="cuda").bfloat16()
    idx = torch.randint(-1, 97, (40, k), device="cuda", dtype=torch.int32)
    out, err = ops.accumulate_rows(src, idx)
    ops.check_error(err)
    want = torch.zeros(40, 7168, device="cuda")
    for j in range(k):
        col = idx[:, j].long()
        ok = col >= 0
        want[ok] += src[col[ok]].float()
    assert (out.float() - want).abs().max().item() <= 1e-2 * want.abs().max().item()


@pytest.mark.parametrize("hidden", [128, 384, 7168])
def test_quant_fp8_matches_the_reference(hidden):
    """kiwi_b200.ops.quant_fp8 (the dispatch kernel's arithmetic in a kernel of
    its own) against the fp32 reference: equal scales; codes equal except where
    a value lies exactly between two e4m3 codes; all-zero blocks get scale 1."""
    from kiwi_b200.models import moe

    torch.manual_seed(hidden)
    x = (torch.randn(37, hidden, device="cuda") * 3).bfloat16()
    x[5] = 0
    codes, scales = ops.quant_fp8(x)
    rc, rs = moe.quant_fp8_codes(x)
    assert codes.dtype == torch.float8_e4m3fn and tuple(scales.shape) == (37, hidden // 128)
    assert torch.allclose(scales, rs, rtol=1e-6, atol=0) and bool((scales[5] == 1).all())
    diff = (codes.float() - rc.float()).abs()
    assert (diff > 0).float().mean().item() < 5e-3
    assert (diff <= torch.maximum(rc.float().abs(), codes.float().abs()) * 0.125 + 2.0 ** -9).all()  # one code


@pytest.mark.parametrize("hidden", [512, 4096, 7168, 80])
def test_quant_nvfp4_matches_the_reference(hidden):
    """kiwi_b200.ops.quant_nvfp4 (the dispatch kernel's NVFP4 arithmetic in a
    kernel of its own) against the fp32 reference: equal row scales, block
    scales and padding; codes equal except where a value lies exactly between
    two e2m1 codes; an all-zero row gets zero scales and codes."""
    from kiwi_b200.models import moe

    torch.manual_seed(hidden + 1)
    x = (torch.randn(41, hidden, device="cuda") * 2).bfloat16()
    x[7] = 0
    codes, scales = ops.quant_nvfp4(x)
    rc, rs = moe.quant_nvfp4_codes(x)
    assert codes.dtype == torch.uint8 and tuple(codes.shape) == (41, hidden // 2)
    assert tuple(scales.shape) == tuple(rs.shape) == (41, moe.nvfp4_scale_bytes(hidden))
    assert torch.equal(scales, rs)
    assert bool((codes[7] == 0).all()) and bool((scales[7] == 0).all())
    d = moe.dequant_nvfp4(codes, scales)
    r = moe.dequant_nvfp4(rc, rs)
    assert (d != r).float().mean().item() < 1e-3
    ref = moe.quant_nvfp4_reference(x)
    assert torch.equal(r, ref)
