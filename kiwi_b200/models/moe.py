"""MoE expert FFN model definitions and fp32 reference implementations.

The benchmark configurations (synthetic seeded data, random-init weights):

* ``deepseek_fp8``  hidden 7168, expert FFN 7168 -> 2048 -> 7168 SwiGLU, 256
  experts, top-8, 1x128 block-scaled FP8 e4m3 dispatch, bf16 compute;
  128 (latency mode) or 4096 (throughput mode) tokens per rank.
* ``nvfp4``  hidden 4096, 64 experts, top-6, NVFP4 dispatch (16-element
  blocks, e4m3 scales), 8192 tokens per rank, Zipf(1.2)-skewed routing.

Weights are N(0, 0.02), drawn per global expert id from its own seeded
generator, so rank r of a world of N holds exactly the experts a world of 1
would hold at the same ids.
"""
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

FP8_MAX = 448.0
FP4_MAX = 6.0
FP4_VALUES = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


@dataclass
class MoEConfig:
    """Shape of one MoE layer and its synthetic workload: hidden size, expert FFN
    width, expert count, top-k, tokens per rank, dispatch wire format
    ("fp8" 1x128 blocks, "nvfp4" 16-element blocks, "none" = bf16), router skew
    (Zipf exponent; 0 = N(0, 1) logits) and seed.  CONFIGS holds the benchmark
    configurations."""
    hidden: int = 7168
    ffn: int = 2048
    num_experts: int = 256
    topk: int = 8
    tokens_per_rank: int = 4096
    quant: str = "fp8"            # "fp8" | "nvfp4" | "none"
    zipf: float = 0.0             # router skew exponent (0 = N(0,1) logits)
    seed: int = 0
    name: str = field(default="deepseek_fp8")

    def flops_per_token(self):
        # top-k experts x (GEMM1 2*H*2F + GEMM2 2*F*H)
        return self.topk * (2 * self.hidden * 2 * self.ffn + 2 * self.ffn * self.hidden)


CONFIGS = {
    "deepseek_fp8": MoEConfig(),
    "deepseek_fp8_latency": MoEConfig(tokens_per_rank=128, name="deepseek_fp8_latency"),
    "nvfp4": MoEConfig(hidden=4096, ffn=1536, num_experts=64, topk=6, tokens_per_rank=8192, quant="nvfp4",
                       zipf=1.2, name="nvfp4"),
}


def expert_weights(cfg, expert, device, dtype=torch.bfloat16, std=0.02):
    """(w1 gate [F, H], w3 up [F, H], w2 down [H, F]) of one global expert id."""
    g = torch.Generator(device=device)
    g.manual_seed(cfg.seed * 1_000_003 + expert)
    w1 = torch.randn(cfg.ffn, cfg.hidden, generator=g, device=device, dtype=torch.float32).mul_(std).to(dtype)
    w3 = torch.randn(cfg.ffn, cfg.hidden, generator=g, device=device, dtype=torch.float32).mul_(std).to(dtype)
    w2 = torch.randn(cfg.hidden, cfg.ffn, generator=g, device=device, dtype=torch.float32).mul_(std).to(dtype)
    return w1, w3, w2


def interleave_gate_up(w1, w3, block=128):
    """Stacks gate and up rows in blocks of `block` rows: [g0, u0, g1, u1, ...],
    the layout the fused SwiGLU epilogue expects (one 256-column accumulator
    tile holds gate rows 128n..128n+127 and the matching up rows)."""
    f, h = w1.shape
    assert f % block == 0
    g = w1.view(f // block, block, h)
    u = w3.view(f // block, block, h)
    return torch.stack([g, u], dim=1).reshape(2 * f, h)


def local_expert_weights(cfg, rank, world, device, dtype=torch.bfloat16):
    """Interleaved w13 [E_local * 2F, H] and w2 [E_local * H, F] of one rank."""
    epr = cfg.num_experts // world
    w13 = torch.empty(epr * 2 * cfg.ffn, cfg.hidden, device=device, dtype=dtype)
    w2 = torch.empty(epr * cfg.hidden, cfg.ffn, device=device, dtype=dtype)
    for j in range(epr):
        a, b, c = expert_weights(cfg, rank * epr + j, device, dtype)
        w13[j * 2 * cfg.ffn:(j + 1) * 2 * cfg.ffn] = interleave_gate_up(a, b)
        w2[j * cfg.hidden:(j + 1) * cfg.hidden] = c
    return w13, w2


def synthetic_inputs(cfg, rank, device, tokens=None, step=0):
    """Seeded activations x ~ N(0,1) (bf16) and router logits (fp32) of one rank.
    With cfg.zipf > 0 the logits get a Zipf(s) popularity bias per expert."""
    t = cfg.tokens_per_rank if tokens is None else tokens
    g = torch.Generator(device=device)
    g.manual_seed((cfg.seed + 1) * 7919 + rank * 104729 + step)
    x = torch.randn(t, cfg.hidden, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
    logits = torch.randn(t, cfg.num_experts, generator=g, device=device, dtype=torch.float32)
    if cfg.zipf > 0:
        ranks = torch.arange(1, cfg.num_experts + 1, device=device, dtype=torch.float32)
        perm = torch.randperm(cfg.num_experts, generator=torch.Generator().manual_seed(cfg.seed)).to(device)
        logits = logits + (cfg.zipf * -torch.log(ranks))[perm] * 2.0
    return x, logits


def route_reference(logits, topk):
    """Top-k experts and softmax over the selected logits (fp32)."""
    v, i = torch.topk(logits.float(), topk, dim=-1)
    return i.to(torch.int32), torch.softmax(v, dim=-1)


# ---------------------------------------------------------------- quantisation


def quant_fp8_codes(x, block=128):
    """1 x `block` FP8 e4m3 quantisation of rows of x, the dispatch wire format:
    (codes float8_e4m3fn [t, h], fp32 scales [t, h / block]) with scale =
    amax / 448 per block (1 for an all-zero block)."""
    t, h = x.shape
    xf = x.float().view(t, h // block, block)
    amax = xf.abs().amax(-1, keepdim=True)
    # Tensor operands keep both divisions IEEE, as on the device (a Python
    # scalar operand makes CUDA multiply by a reciprocal instead).
    fmax = torch.full_like(amax, FP8_MAX)
    scale = torch.where(amax > 0, amax / fmax, torch.ones_like(amax))
    inv = torch.where(amax > 0, fmax / amax, torch.zeros_like(amax))  # then multiply by it, as on the device
    q = (xf * inv).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q.view(t, h), scale.view(t, h // block)


def quant_fp8_reference(x, block=128):
    """1 x `block` FP8 e4m3 quantise-dequantise of rows of x (fp32 scale = amax / 448)."""
    t, h = x.shape
    q, scale = quant_fp8_codes(x, block)
    return (q.float().view(t, h // block, block) * scale.unsqueeze(-1)).view(t, h)


def _round_fp4(v):
    """Round-to-nearest-even onto the e2m1 grid (saturating at 6)."""
    codes = fp4_codes(v).long()
    mag = FP4_VALUES.to(v.device)[codes & 7]
    return torch.where(codes >= 8, -mag, mag)


def fp4_codes(v):
    """e2m1 codes (uint8, 0..15: sign in bit 3, the index into FP4_VALUES below
    it) of v rounded to nearest-even on the e2m1 grid, saturating at +-6."""
    grid = FP4_VALUES.to(v.device)
    a = v.float().abs().clamp(max=FP4_MAX)
    d = (a.unsqueeze(-1) - grid).abs()
    idx = torch.argmin(d + (torch.arange(len(grid), device=v.device) % 2) * 1e-6, dim=-1)
    return (idx | ((v < 0).to(idx.dtype) << 3)).to(torch.uint8)


def fp4_pack(codes):
    """[..., 2m] e2m1 codes -> [..., m] bytes, element 2i in the low nibble."""
    c = codes.to(torch.uint8)
    return c[..., 0::2] | (c[..., 1::2] << 4)


def fp4_unpack(packed):
    """[..., m] packed e2m1 bytes -> [..., 2m] fp32 values (inverse of fp4_pack)."""
    b = packed.view(torch.uint8)
    codes = torch.stack([b & 0xF, b >> 4], dim=-1).flatten(-2).long()
    mag = FP4_VALUES.to(b.device)[codes & 7]
    return torch.where(codes >= 8, -mag, mag)


def nvfp4_scale_bytes(hidden, block=16):
    """Scale bytes of one NVFP4 row on the wire: fp32 row scale + one e4m3 byte
    per block, padded to 16 bytes."""
    return (4 + hidden // block + 15) // 16 * 16


def _nvfp4_parts(x, block=16):
    """(row_scale [t, 1], e4m3 block scales [t, h/block, 1], per-element scale, e2m1 codes [t, h])."""
    t, h = x.shape
    xf = x.float()
    row_amax = xf.abs().amax(-1, keepdim=True)
    # A tensor divisor keeps this an IEEE division (a Python scalar divisor
    # becomes a multiply by its reciprocal on CUDA), as the kernels divide.
    row_scale = torch.where(row_amax > 0, row_amax / torch.full_like(row_amax, FP8_MAX * FP4_MAX),
                            torch.zeros_like(row_amax))
    xb = xf.view(t, h // block, block)
    bamax = xb.abs().amax(-1, keepdim=True)
    s = torch.where(row_scale[:, :, None] > 0, bamax / (FP4_MAX * row_scale[:, :, None]), torch.zeros_like(bamax))
    s8 = s.clamp(max=FP8_MAX).to(torch.float8_e4m3fn)
    sdec = s8.float() * row_scale[:, :, None]
    inv = torch.where(sdec > 0, 1.0 / sdec, torch.zeros_like(sdec))
    return row_scale, s8, sdec, fp4_codes(xb * inv).view(t, h)


def quant_nvfp4_codes(x, block=16):
    """NVFP4 wire format of rows x [t, h]: (packed e2m1 codes uint8 [t, h / 2],
    element 2i in the low nibble; scale bytes uint8 [t, nvfp4_scale_bytes(h)] =
    fp32 row scale amax / (448 * 6), then one e4m3 block scale per `block`
    elements relative to it, zero padding)."""
    t, h = x.shape
    row_scale, s8, _, codes = _nvfp4_parts(x, block)
    sc = torch.zeros(t, nvfp4_scale_bytes(h, block), dtype=torch.uint8, device=x.device)
    sc[:, :4] = row_scale.contiguous().view(torch.uint8).view(t, 4)
    sc[:, 4:4 + h // block] = s8.view(t, h // block).view(torch.uint8)
    return fp4_pack(codes), sc


def dequant_nvfp4(codes, scales, block=16):
    """fp32 rows [t, h] of the NVFP4 wire format (inverse of quant_nvfp4_codes)."""
    t, h = codes.shape[0], codes.shape[1] * 2
    row_scale = scales[:, :4].contiguous().view(torch.float32)                    # [t, 1]
    s = scales[:, 4:4 + h // block].contiguous().view(torch.float8_e4m3fn).float() * row_scale
    return (fp4_unpack(codes).view(t, h // block, block) * s[:, :, None]).view(t, h)


def quant_nvfp4_reference(x, block=16):
    """NVFP4 quantise-dequantise: per-row fp32 scale amax/(448*6), e4m3 block
    scales per `block` elements, e2m1 values."""
    t, h = x.shape
    _, _, sdec, codes = _nvfp4_parts(x, block)
    q = fp4_unpack(fp4_pack(codes)).view(t, h // block, block)
    return (q * sdec).view(t, h)


def dispatch_reference(x, quant):
    """What the dispatch kernel delivers for rows `x` in wire format `quant`,
    dequantised to fp32 (the reference the receive-side tests compare with)."""
    if quant == "fp8":
        return quant_fp8_reference(x)
    if quant in ("nvfp4", "fp4"):
        return quant_nvfp4_reference(x)
    return x.float()


# ---------------------------------------------------------------- reference layer


def moe_reference(cfg, x, idx, w, world=1, device=None, quant=None, expert_ids=None):
    """fp32 reference of the whole layer for the tokens of one rank: dispatch
    quantisation (as the wire format does), expert SwiGLU FFN in fp32 on the
    bf16 weights, routing-weighted sum over the top-k experts."""
    device = device or x.device
    quant = cfg.quant if quant is None else quant
    xq = dispatch_reference(x, quant)
    out = torch.zeros(x.shape[0], cfg.hidden, device=device, dtype=torch.float32)
    experts = torch.unique(idx).tolist() if expert_ids is None else expert_ids
    for e in experts:
        rows, slot = (idx == e).nonzero(as_tuple=True)
        if rows.numel() == 0:
            continue
        w1, w3, w2 = expert_weights(cfg, int(e), device)
        a = xq[rows].bfloat16().float()
        hdn = F.silu(a @ w1.float().t()) * (a @ w3.float().t())
        hdn = hdn.bfloat16().float()
        y = hdn @ w2.float().t()
        out.index_add_(0, rows, y * w[rows, slot].float()[:, None])
    return out
