"""The fused EP MoE layer on one B200 (world of 1: every store goes through
the same NVLink-path code into the local heap) vs the fp32 reference."""
import pytest
import torch

import kiwi_b200
from kiwi_b200 import ops
from kiwi_b200.models import moe
from kiwi_b200.parallel.ep import EpDispatchCombine, ExpertParallelMoE

pytestmark = pytest.mark.gpu


def small_cfg(quant, tokens=200, hidden=1024, ffn=256, experts=16, topk=4, zipf=0.0):
    return moe.MoEConfig(hidden=hidden, ffn=ffn, num_experts=experts, topk=topk, tokens_per_rank=tokens,
                         quant=quant, zipf=zipf, name="test")


def _check(layer, cfg, x, logits, out, rel=2e-2):
    torch.cuda.synchronize()
    layer.check()
    idx, w = moe.route_reference(logits, cfg.topk)
    ref = moe.moe_reference(cfg, x, idx, w, device=x.device)
    got = out.float()
    scale = ref.abs().max().item()
    err = (got - ref).abs().max().item()
    assert err <= rel * scale + 1e-3, (err, scale)


@pytest.mark.parametrize("fused,gather", [(True, True), (False, True), (True, False), (False, False)])
@pytest.mark.parametrize("quant", ["fp8", "nvfp4", "none"])
def test_layer_matches_reference(quant, fused, gather):
    """fused=True: GEMM2's epilogue stores the weighted rows into the token
    owners' top-k slots (fused combine); False: GEMM2, combine send, receive.
    gather=True: GEMM1 gathers and dequantises its A rows from the receive
    slots; False: expert-major bf16 rows are written first, TMA loads them."""
    cfg = small_cfg(quant)
    layer = ExpertParallelMoE(cfg)
    layer.native.fused_combine = fused
    layer.native.gather_a = gather
    # NVFP4 keeps one mantissa bit: a single rounding disagreement between two
    # correct quantisers moves an output by a visible fraction of its range.
    rel = 5e-2 if quant == "nvfp4" else 2e-2
    for step in range(3):  # several rounds: epochs advance, slots reused
        x, logits = moe.synthetic_inputs(cfg, 0, "cuda", step=step)
        out = layer(x, logits).clone()
        _check(layer, cfg, x, logits, out, rel)


def _hidden_by_row(layer, cfg):
    """GEMM1 output rows keyed by (local expert, source slot), sorted: row
    order inside an expert follows atomics and may differ between rounds."""
    n = int(layer.expert_counts.sum().item())
    offs = layer.native.expert_offsets.long()
    pos = torch.arange(n, device=offs.device)
    expert = torch.searchsorted(offs[1:], pos, right=True)
    key = expert * (1 << 32) + layer.native.pair_slot[:n].long()
    order = torch.argsort(key)
    return key[order], layer.native.expert_hidden[:n][order].clone()


@pytest.mark.parametrize("quant", ["fp8", "nvfp4"])
def test_gathered_gemm1_equals_materialised_rows(quant):
    """GEMM1 fed by the gathering producer (dequantised in shared memory)
    gives bit-identical rows to GEMM1 over the receive kernel's bf16 rows."""
    cfg = small_cfg(quant, tokens=200, zipf=1.2)
    layer = ExpertParallelMoE(cfg)
    x, logits = moe.synthetic_inputs(cfg, 0, "cuda")
    out = {}
    for gather in (False, True):
        layer.native.gather_a = gather
        layer(x, logits)
        torch.cuda.synchronize()
        layer.check()
        out[gather] = _hidden_by_row(layer, cfg)
    assert torch.equal(out[False][0], out[True][0])
    assert torch.equal(out[False][1], out[True][1])


@pytest.mark.parametrize("quant", ["fp8", "nvfp4", "none"])
def test_dispatched_rows_match_reference_quantisation(quant):
    """Each expert-major row the receive side produced equals the reference
    quantise-dequantise of its source token (bf16-rounded)."""
    cfg = small_cfg(quant, tokens=64)
    layer = ExpertParallelMoE(cfg)
    layer.native.gather_a = False  # materialise the expert-major rows
    x, logits = moe.synthetic_inputs(cfg, 0, "cuda")
    layer(x, logits)
    torch.cuda.synchronize()
    n = int(layer.expert_counts.sum().item())
    rows = layer.native.expert_input[:n].float()
    tok = (layer.native.pair_slot[:n] % cfg.tokens_per_rank).long()
    ref = moe.dispatch_reference(x, quant).bfloat16().float()[tok]
    # Elements may land one quantisation step apart where the scaled value sits on
    # a rounding boundary (x * (448 / amax) in the kernel vs the reference's
    # fp32 arithmetic); anything more than a tiny fraction is a layout bug.
    bad = (rows - ref).abs() > 1e-6 + 1e-2 * ref.abs()
    assert bad.float().mean().item() < 5e-3, (bad.float().mean().item(), (rows - ref).abs().max().item())


def test_routing_kernel_matches_topk():
    cfg = small_cfg("fp8", tokens=300, experts=64, topk=6)
    _, logits = moe.synthetic_inputs(cfg, 0, "cuda")
    idx = torch.empty(300, 6, dtype=torch.int32, device="cuda")
    w = torch.empty(300, 6, dtype=torch.float32, device="cuda")
    kiwi_b200.native().ep.route(logits, 6, idx, w)
    ridx, rw = moe.route_reference(logits, 6)
    assert torch.equal(idx, ridx)
    assert torch.allclose(w, rw, atol=1e-6)


def test_expert_counts_and_partial_token_counts():
    cfg = small_cfg("fp8", tokens=256, experts=16, topk=4)
    layer = ExpertParallelMoE(cfg)
    x, logits = moe.synthetic_inputs(cfg, 0, "cuda", tokens=77)
    out = layer(x, logits).clone()
    _check(layer, cfg, x, logits, out)
    idx, _ = moe.route_reference(logits, 4)
    assert torch.equal(layer.expert_counts.cpu(), torch.bincount(idx.flatten().long(), minlength=16).int().cpu())


def test_zero_tokens_round():
    cfg = small_cfg("fp8", tokens=64)
    layer = ExpertParallelMoE(cfg)
    x, logits = moe.synthetic_inputs(cfg, 0, "cuda", tokens=0)
    out = layer(x, logits)
    torch.cuda.synchronize()
    layer.check()
    assert out.shape == (0, cfg.hidden)
    x, logits = moe.synthetic_inputs(cfg, 0, "cuda", tokens=64)
    _check(layer, cfg, x, logits, layer(x, logits).clone())


def test_skewed_routing_and_cuda_graph_replay():
    cfg = small_cfg("fp8", tokens=128, zipf=1.2)
    layer = ExpertParallelMoE(cfg)
    x, logits = moe.synthetic_inputs(cfg, 0, "cuda")
    layer(x, logits)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = layer(x, logits)
    for step in range(3):
        x2, l2 = moe.synthetic_inputs(cfg, 0, "cuda", step=step + 10)
        x.copy_(x2)
        logits.copy_(l2)
        g.replay()
        _check(layer, cfg, x, logits, out.clone())


def test_transport_only_dispatch_combine():
    t = EpDispatchCombine(hidden=512, num_experts=8, topk=2, max_tokens=64, quant="none")
    x = torch.randn(64, 512, device="cuda").bfloat16()
    logits = torch.randn(64, 8, device="cuda")
    idx, w = moe.route_reference(logits, 2)
    rows, counts, slots, weights = t.dispatch(x, w, idx)
    torch.cuda.synchronize()
    n = int(counts.sum().item())
    assert n == 64 * 2
    # each received row is its token's row; combine of weight*row must give sum_k w_k * x
    tok = (slots[:n] % 64).long()
    assert torch.equal(rows[:n], x[tok])
    out = t.combine(rows[:n].float().mul(weights[:n, None]).bfloat16())
    torch.cuda.synchronize()
    ref = x.float() * w.sum(-1, keepdim=True)
    assert (out.float() - ref).abs().max().item() < 3e-2


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float8_e4m3fn])
def test_kiwi_ep_op_contract(dtype):
    """Reference/MORI contract: received rows in (source, token) order; combine
    returns each row to its token and sums them without routing weights."""
    from kiwi_b200.parallel.ep import KiwiEpOp

    op = KiwiEpOp(hidden_dim=512, topk=3, num_experts_per_rank=8, max_num_inp_token_per_rank=40,
                  dispatch_dtype=dtype)
    x = torch.randn(40, 512, device="cuda").bfloat16()
    logits = torch.randn(40, 8, device="cuda")
    idx, w = moe.route_reference(logits, 3)
    rows, ow, sc, oidx, cnt = op.dispatch(x, w, None, idx)
    torch.cuda.synchronize()
    op.check()
    n = int(cnt.item())
    assert n == 40  # world of 1: every token arrives once
    pos = op.get_dispatch_src_token_pos()[:n].long()
    assert torch.equal(pos, torch.arange(40, device="cuda"))
    assert torch.equal(oidx[:n], idx) and torch.allclose(ow[:n], w)
    if dtype == torch.bfloat16:
        assert torch.equal(rows[:n], x)
        deq = rows[:n].float()
    else:
        deq = (rows[:n].float().view(n, 4, 128) * sc[:n].view(torch.float32)[:, :4, None]).view(n, 512)
        ref = moe.quant_fp8_reference(x)
        # The kernel and the reference may round a value lying exactly between
        # two e4m3 codes differently (one code apart); everything else matches.
        diff = (deq - ref).abs()
        assert (diff > 1e-6).float().mean().item() < 5e-3, (diff > 1e-6).sum().item()
        assert (diff <= ref.abs() * 0.125 + 1e-6).all()
    out, _ = op.combine(deq.bfloat16(), None, idx)
    torch.cuda.synchronize()
    op.check()
    assert torch.equal(out, deq.bfloat16())


def test_kiwi_ep_op_token_sweep():
    """One op, rounds of 1 to max_num_inp_token_per_rank tokens in a row (the
    reference's 1..256 token sweeps): every round delivers exactly its own
    tokens, in order, and combines them back, so no round reads a stale slot."""
    from kiwi_b200.parallel.ep import KiwiEpOp

    op = KiwiEpOp(hidden_dim=256, topk=2, num_experts_per_rank=4, max_num_inp_token_per_rank=256)
    for i, t in enumerate((1, 2, 31, 128, 255, 256, 7)):
        g = torch.Generator(device="cuda").manual_seed(i)
        x = torch.randn(t, 256, device="cuda", generator=g).bfloat16()
        idx, w = moe.route_reference(torch.randn(t, 4, device="cuda", generator=g), 2)
        rows, ow, _, oidx, cnt = op.dispatch(x, w, None, idx)
        torch.cuda.synchronize()
        op.check()
        n = int(cnt.item())
        assert n == t and torch.equal(rows[:n], x) and torch.equal(oidx[:n], idx), (t, n)
        out, _ = op.combine(rows[:n].clone(), None, idx)
        torch.cuda.synchronize()
        op.check()
        assert torch.equal(out[:t], x), t
        op.reset()


@pytest.mark.parametrize("fused", [True, False])
def test_layer_with_2sm_gemm(fused):
    """Both GEMMs on the 2-SM (256-row tile) kernels: GEMM2 with the NVLink
    scatter epilogue of the fused combine, or plain for the unfused one."""
    cfg = small_cfg("fp8", tokens=300, experts=8)
    layer = ExpertParallelMoE(cfg)
    layer.native.gemm_pair = True
    layer.native.fused_combine = fused
    x, logits = moe.synthetic_inputs(cfg, 0, "cuda")
    _check(layer, cfg, x, logits, layer(x, logits).clone())


@pytest.mark.parametrize("fused", [True, False])
def test_layer_with_2sm_gemm2_only(fused):
    """gemm2_pair: GEMM1 on the 1-SM kernel (128-row tiles), GEMM2 on the 2-SM
    kernel (256-row tiles, scatter epilogue when fused); each GEMM's tile
    schedule uses its own kernel's tile height.  Ragged row counts."""
    cfg = small_cfg("fp8", tokens=700, experts=8)
    layer = ExpertParallelMoE(cfg)
    layer.native.gemm2_pair = True
    layer.native.fused_combine = fused
    for t in (700, 90):
        x, logits = moe.synthetic_inputs(cfg, 0, "cuda", tokens=t, step=t)
        out = layer(x, logits).clone()
        assert layer.native.gemm2_pair_in_use and not layer.native.gemm_pair_in_use
        _check(layer, cfg, x, logits, out)


@pytest.mark.parametrize("fused", [True, False])
def test_layer_m64_tail_tiles_are_bit_identical(fused):
    """gemm_m64_tails (default on) runs M = 64 MMAs on the 1-SM GEMM tiles with
    at most 64 rows of their expert left; the layer's output equals the
    M = 128 run bit for bit and the fp32 reference within tolerance."""
    cfg = small_cfg("fp8", tokens=600, experts=8)
    layer = ExpertParallelMoE(cfg)
    layer.native.fused_combine = fused
    assert layer.native.gemm_m64_tails
    x, logits = moe.synthetic_inputs(cfg, 0, "cuda")
    on = layer(x, logits).clone()
    assert any(c % 128 and c % 128 <= 64 for c in layer.expert_counts.tolist())
    layer.native.gemm_m64_tails = False
    off = layer(x, logits).clone()
    torch.cuda.synchronize()
    assert torch.equal(on, off)
    _check(layer, cfg, x, logits, on)


@pytest.mark.parametrize("pair", [False, True])
def test_layer_blocked_weights_are_bit_identical(pair):
    """weight_layout="blocked" (the default: the layer keeps w13 / w2 as one
    contiguous 256 x 64 box per TMA load) gives the row-major layer's output
    bit for bit, with the 1-SM and the 2-SM GEMMs (fused combine)."""
    cfg = small_cfg("fp8", tokens=400, experts=8)
    rows = ExpertParallelMoE(cfg, weight_layout="rows")
    blocked = ExpertParallelMoE(cfg)
    assert blocked.weight_layout == "blocked" and blocked.w13.shape[1] == 64
    for layer in (rows, blocked):
        layer.native.gemm_pair = pair
    x, logits = moe.synthetic_inputs(cfg, 0, "cuda")
    a = rows(x, logits).clone()
    b = blocked(x, logits).clone()
    torch.cuda.synchronize()
    rows.check()
    blocked.check()
    assert torch.equal(a, b)
    _check(blocked, cfg, x, logits, b)


@pytest.mark.parametrize("fused", [True, False])
def test_split_gemms_match_reference(fused):
    """gemm_split runs each GEMM as a 2-SM pass over every expert's full 256-row
    tiles plus a 1-SM pass over its tail (GEMM2 with the NVLink scatter
    epilogue in both passes, the second one signalling the round).  Row counts
    are ragged (routing from random logits), so experts have tails."""
    cfg = small_cfg("fp8", tokens=1536, experts=8)
    layer = ExpertParallelMoE(cfg)
    layer.native.fused_combine = fused
    layer.native.gemm_split = True
    for t in (1536, 200, 1024):
        x, logits = moe.synthetic_inputs(cfg, 0, "cuda", tokens=t, step=t)
        out = layer(x, logits).clone()
        assert layer.native.gemm_split_in_use and not layer.native.gemm_pair_in_use
        counts = layer.expert_counts.tolist()
        assert any(c % 256 for c in counts)
        _check(layer, cfg, x, logits, out)


def test_2sm_gemms_chosen_from_4096_rows_per_expert():
    """With the defaults a round runs the 2-SM GEMMs when it expects at least
    4096 rows per local expert, the 1-SM ones otherwise; both match the
    reference."""
    cfg = small_cfg("fp8", tokens=8192, experts=8)
    layer = ExpertParallelMoE(cfg)
    assert layer.native.gemm_pair_auto and not layer.native.gemm_pair and not layer.native.gemm_split
    for t, pair in ((8192, True), (1024, False)):
        x, logits = moe.synthetic_inputs(cfg, 0, "cuda", tokens=t, step=t)
        out = layer(x, logits).clone()
        assert layer.native.gemm_pair_in_use == pair and not layer.native.gemm_split_in_use
        g = torch.Generator(device="cpu").manual_seed(t)
        pick = torch.randperm(t, generator=g)[:64].to(x.device)
        _check(layer, cfg, x[pick], logits[pick], out[pick])


@pytest.mark.parametrize("quant", ["fp8", "nvfp4"])
def test_rounds_in_flight_match_reference(quant):
    """Two rounds in flight: five rounds with different inputs submitted back
    to back on the two slots' streams, each output checked against the fp32
    reference once waited for; forward() on the same layer stays synchronous."""
    cfg = small_cfg(quant, tokens=160)
    layer = ExpertParallelMoE(cfg, in_flight=2)
    ins = [moe.synthetic_inputs(cfg, 0, "cuda", step=i, tokens=160 - 8 * i) for i in range(5)]
    outs = [torch.empty(x.shape[0], cfg.hidden, dtype=torch.bfloat16, device="cuda") for x, _ in ins]
    pend = [layer.submit(x, lg, out=o) for (x, lg), o in zip(ins, outs)]
    for p in pend:
        layer.wait(p)
    for (x, lg), o in zip(ins, outs):
        _check(layer, cfg, x, lg, o, rel=5e-2 if quant == "nvfp4" else 2e-2)
    x, lg = ins[0]
    _check(layer, cfg, x, lg, layer(x, lg).clone(), rel=5e-2 if quant == "nvfp4" else 2e-2)


_FP4 = torch.float4_e2m1fn_x2


@pytest.mark.parametrize("comb", ["f32", "fp8", "fp4", "bf16"])
def test_kiwi_ep_op_combine_dtypes_and_weight_sums(comb):
    """Combine in every dtype the reference accepts (float32, bfloat16, FP8
    e4m3 codes, packed FP4 e2m1 codes), with the rows' top-k weights travelling
    back and summed per token.  On one rank every token returns exactly one
    row, so the output is that row (codes re-encoded exactly) and the weight
    sum is the row's own weights."""
    from kiwi_b200.models.moe import fp4_codes, fp4_pack, fp4_unpack
    from kiwi_b200.parallel.ep import KiwiEpOp

    dt, fmt = {"f32": (torch.float32, "none"), "bf16": (torch.bfloat16, "none"),
               "fp8": (torch.float8_e4m3fn, "fp8"), "fp4": (_FP4, "fp4")}[comb]
    op = KiwiEpOp(hidden_dim=512, topk=3, num_experts_per_rank=8, max_num_inp_token_per_rank=40,
                  combine_dtype=dt, combine_quant_format=fmt)
    torch.manual_seed(7)
    x = torch.randn(37, 512, device="cuda").bfloat16()
    idx, w = moe.route_reference(torch.randn(37, 8, device="cuda"), 3)
    rows, ow, _, oidx, cnt = op.dispatch(x, w, None, idx)
    torch.cuda.synchronize()
    n = int(cnt.item())
    assert n == 37
    y = rows[:n].float() * 3.0                      # values past the FP8 / FP4 ranges too
    if comb == "fp4":
        inp = fp4_pack(fp4_codes(y)).view(_FP4)
        expect = fp4_unpack(inp)
    elif comb == "fp8":
        inp = y.clamp(-448, 448).to(torch.float8_e4m3fn)
        expect = inp.float()
    else:
        inp = y.to(dt)
        expect = inp.float()
    out, out_w = op.combine(inp, ow[:n], oidx[:n])
    torch.cuda.synchronize()
    op.check()
    assert out.dtype == dt and out.shape[0] == 37
    got = fp4_unpack(out) if comb == "fp4" else out.float()
    assert torch.equal(got, expect)
    assert out_w is not None and torch.equal(out_w, ow[:n])
    out2, none_w = op.combine(inp, None, oidx[:n])
    torch.cuda.synchronize()
    assert none_w is None and torch.equal(fp4_unpack(out2) if comb == "fp4" else out2.float(), expect)


def test_kiwi_ep_op_pre_quantised_fp8_dispatch():
    """FP8 codes the caller quantised, with its own per-token scales
    (dispatch_scale_dim x dispatch_scale_type_size bytes), travel unchanged:
    the received codes and scales equal the sent ones (the reference's
    pre-quantised contract)."""
    from kiwi_b200.parallel.ep import KiwiEpOp

    op = KiwiEpOp(hidden_dim=512, topk=2, num_experts_per_rank=8, max_num_inp_token_per_rank=32,
                  dispatch_dtype=torch.float8_e4m3fn, dispatch_quant_format="fp8", dispatch_scale_dim=16,
                  dispatch_scale_type_size=4)
    torch.manual_seed(3)
    codes = (torch.randn(32, 512, device="cuda") * 40).to(torch.float8_e4m3fn)
    scales = torch.rand(32, 16, device="cuda")      # e.g. 1x32 blocks, the caller's choice
    idx, w = moe.route_reference(torch.randn(32, 8, device="cuda"), 2)
    rows, ow, sc, oidx, cnt = op.dispatch(codes, w, scales, idx)
    torch.cuda.synchronize()
    op.check()
    n = int(cnt.item())
    assert n == 32
    assert rows.dtype == torch.float8_e4m3fn and torch.equal(rows[:n].view(torch.uint8), codes.view(torch.uint8))
    assert sc.dtype == torch.float32 and tuple(sc.shape[1:]) == (16,) and torch.equal(sc[:n], scales)
    with pytest.raises(ValueError):
        op.dispatch(codes, w, scales[:, :8], idx)   # not the configured scale size


def test_kiwi_ep_op_pre_quantised_fp4_dispatch_and_own_quantisation():
    """An FP4 op takes packed e2m1 rows [T, hidden / 2] with the caller's scale
    bytes unchanged, and bf16 rows it quantises itself (scale bytes of the
    NVLink wire format); bf16 rows with caller scales are refused there."""
    from kiwi_b200.parallel.ep import KiwiEpOp

    op = KiwiEpOp(hidden_dim=512, topk=2, num_experts_per_rank=8, max_num_inp_token_per_rank=32,
                  dispatch_dtype=torch.uint8, dispatch_quant_format="fp4", dispatch_scale_dim=32,
                  dispatch_scale_type_size=1, dispatch_scale_dtype=torch.uint8)
    torch.manual_seed(5)
    packed = torch.randint(0, 256, (32, 256), dtype=torch.uint8, device="cuda")
    sbytes = torch.randint(0, 256, (32, 32), dtype=torch.uint8, device="cuda")
    idx, w = moe.route_reference(torch.randn(32, 8, device="cuda"), 2)
    rows, _, sc, _, cnt = op.dispatch(packed.view(_FP4), w, sbytes, idx)
    torch.cuda.synchronize()
    op.check()
    n = int(cnt.item())
    assert torch.equal(rows[:n].view(torch.uint8), packed) and torch.equal(sc[:n], sbytes)
    x = torch.randn(32, 512, device="cuda").bfloat16()
    rows, _, sc, _, cnt = op.dispatch(x, w, None, idx)
    torch.cuda.synchronize()
    op.check()
    ref_codes, ref_sc = ops.quant_nvfp4(x)
    assert torch.equal(rows[:n].view(torch.uint8), ref_codes)
    assert torch.equal(sc[:n, :ref_sc.shape[1]], ref_sc)
    with pytest.raises(ValueError):
        op.dispatch(x, w, sbytes, idx)


def test_kiwi_ep_op_bf16_rows_carry_caller_scales():
    """A bf16 op carries the caller's per-token scales next to the rows."""
    from kiwi_b200.parallel.ep import KiwiEpOp

    op = KiwiEpOp(hidden_dim=256, topk=2, num_experts_per_rank=4, max_num_inp_token_per_rank=16,
                  dispatch_scale_dim=3, dispatch_scale_type_size=4)
    x = torch.randn(16, 256, device="cuda").bfloat16()
    scales = torch.randn(16, 3, device="cuda")
    idx, w = moe.route_reference(torch.randn(16, 4, device="cuda"), 2)
    rows, _, sc, _, cnt = op.dispatch(x, w, scales, idx)
    torch.cuda.synchronize()
    op.check()
    n = int(cnt.item())
    assert torch.equal(rows[:n], x) and torch.equal(sc[:n], scales)


@pytest.mark.filterwarnings("ignore:The CUDA Graph is empty")
@pytest.mark.parametrize("fused", [True, False])
def test_debug_timing_spans_every_kernel_of_a_round(fused):
    """Opt-in phase timing: each kernel's span (first block start, last warp
    end) is recorded per round, in stream order, and the receive-side flag
    waits sit inside their kernels."""
    cfg = small_cfg("fp8", tokens=128)
    layer = ExpertParallelMoE(cfg)
    layer.native.fused_combine = fused
    x, logits = moe.synthetic_inputs(cfg, 0, "cuda")
    layer(x, logits)
    snap = layer.get_debug_timing_snapshot()
    assert not snap["enabled"] and not any(snap["time_ticks"])
    layer.set_debug_timing_enabled(True)
    for step in range(2):  # the second round must not keep the first round's stamps
        x, logits = moe.synthetic_inputs(cfg, 0, "cuda", step=step)
        out = layer(x, logits).clone()
        snap = layer.get_debug_timing_snapshot()
    _check(layer, cfg, x, logits, out)
    ph = snap["phases"]
    order = ["route", "begin", "dispatch", "dispatch_wait", "recv_count", "recv_assign", "recv_copy", "gemm1",
             "gemm2"]
    order += ["combine_wait", "combine_recv"] if fused else ["combine_send", "combine_wait", "combine_recv"]
    assert set(order) <= set(ph), sorted(ph)
    slack = 2.0  # us: %globaltimer granularity
    for a, b in zip(order, order[1:]):
        assert ph[a]["end_us"] <= ph[b]["start_us"] + slack, (a, b, ph[a], ph[b])
    for name in order:
        assert ph[name]["us"] >= 0
    for name in ("dispatch_wait", "combine_wait"):  # the flag waits run in a 32-thread kernel of their own
        assert "wait_us" in ph[name]
        assert ph[name]["start_us"] - slack <= ph[name]["wait_start_us"] <= ph[name]["wait_end_us"] + slack
        assert ph[name]["wait_end_us"] <= ph[name]["end_us"] + slack
    span = ph[order[-1]]["end_us"] - ph["route"]["start_us"]
    assert 0 < span < 1e6
    meta = dict(zip(snap["meta_names"], snap["meta"]))
    assert meta["world"] == 1 and meta["tokens"] == 128 and meta["recv_tokens"] == 128
    assert meta["expert_rows"] == 128 * cfg.topk and meta["fused_combine"] == int(fused)
    # a graph capture must not read the buffer
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        with pytest.raises(RuntimeError):
            layer.get_debug_timing_snapshot()
    layer.set_debug_timing_enabled(False)
    assert not layer.debug_timing_enabled


def test_debug_timing_of_the_transport_op():
    from kiwi_b200.parallel.ep import KiwiEpOp

    op = KiwiEpOp(hidden_dim=512, topk=2, num_experts_per_rank=8, max_num_inp_token_per_rank=32)
    op.set_debug_timing_enabled(True)
    x = torch.randn(32, 512, device="cuda").bfloat16()
    idx, w = moe.route_reference(torch.randn(32, 8, device="cuda"), 2)
    rows, _, _, _, cnt = op.dispatch(x, w, None, idx)
    op.combine(rows[:32].clone(), None, idx)
    snap = op.get_debug_timing_snapshot()
    op.check()
    ph = snap["phases"]
    for name in ("dispatch", "recv_count", "recv_compact", "gather_rows", "combine_rows", "combine_recv"):
        assert name in ph, sorted(ph)
    assert ph["dispatch"]["end_us"] <= ph["combine_recv"]["start_us"] + 2.0


@pytest.mark.filterwarnings("ignore:The CUDA Graph is empty")
def test_kiwi_ep_op_reference_accessors():
    """launch_policy, the registered combine-input buffer (combine straight
    from it), source positions and reset() refused during graph capture."""
    from kiwi_b200.parallel.ep import KiwiEpOp

    op = KiwiEpOp(hidden_dim=256, topk=2, num_experts_per_rank=4, max_num_inp_token_per_rank=16)
    pol = op.launch_policy(16)
    assert pol["num_blocks"] > 0 and pol["transport"] == "nvlink" and pol["num_tokens"] == 16
    buf = op.get_registered_combine_input_buffer(torch.bfloat16)
    assert tuple(buf.shape) == (16, 256) and buf.data_ptr() == op.get_registered_combine_input_buffer().data_ptr()
    x = torch.randn(16, 256, device="cuda").bfloat16()
    idx, w = moe.route_reference(torch.randn(16, 4, device="cuda"), 2)
    rows, _, _, _, cnt = op.dispatch(x, w, None, idx)
    n = int(cnt.item())
    assert n == 16
    pos = op.get_dispatch_src_token_pos()
    assert [op.decode_send_flat_idx(p) for p in pos.tolist()] == [(0, t) for t in range(16)]
    buf[:n].copy_(rows[:n])
    out, _ = op.combine(buf, None, idx)
    torch.cuda.synchronize()
    op.check()
    assert torch.equal(out, x)  # world of 1: one row per token comes back unchanged
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        with pytest.raises(RuntimeError):
            op.reset()
    op.reset()


def test_collective_op_matches_the_nvlink_op():
    """CollectiveEpOp (all-to-all transport, for ranks across nodes) and
    KiwiEpOp (NVLink stores) deliver the same rows, ids, weights and source
    positions, and combine to the same sums, on one GPU."""
    from kiwi_b200.parallel.ep import KiwiEpOp
    from kiwi_b200.parallel.ep_collective import CollectiveEpOp

    kw = dict(hidden_dim=512, topk=2, num_experts_per_rank=8, max_num_inp_token_per_rank=32)
    a, b = KiwiEpOp(**kw), CollectiveEpOp(**kw)
    torch.manual_seed(3)
    x = torch.randn(32, 512, device="cuda").bfloat16()
    idx, w = moe.route_reference(torch.randn(32, 8, device="cuda"), 2)
    ra, wa, _, ia, ca = a.dispatch(x, w, None, idx)
    rb, wb, _, ib, cb = b.dispatch(x, w, None, idx)
    n = int(ca.item())
    assert n == int(cb.item()) == 32
    assert torch.equal(ra[:n], rb[:n]) and torch.equal(ia[:n], ib[:n]) and torch.allclose(wa[:n], wb[:n])
    assert a.get_dispatch_src_token_pos().tolist() == b.get_dispatch_src_token_pos().tolist()
    oa, _ = a.combine(ra[:n].clone(), None, idx)
    ob, _ = b.combine(rb[:n].clone(), None, idx)
    torch.cuda.synchronize()
    a.check()
    assert torch.equal(oa, ob) and torch.equal(oa, x)


@pytest.mark.parametrize("quant", ["none", "fp8"])
def test_collective_moe_layer_on_one_gpu(quant):
    """CollectiveMoE (all-to-all transport + the tcgen05 expert FFN) against the
    fp32 layer reference."""
    from kiwi_b200.parallel.ep_collective import CollectiveMoE

    cfg = moe.MoEConfig(hidden=512, ffn=256, num_experts=8, topk=2, tokens_per_rank=64, quant=quant, name="t")
    layer = CollectiveMoE(cfg)
    assert layer.device.type == "cuda"
    for step in range(2):
        x, logits = moe.synthetic_inputs(cfg, 0, "cuda", tokens=64 - 20 * step, step=step)
        out = layer(x, logits)
        torch.cuda.synchronize()
        layer.check()
        idx, w = moe.route_reference(logits, cfg.topk)
        ref = moe.moe_reference(cfg, x, idx, w, device=x.device)
        assert (out.float() - ref).abs().max().item() <= 2e-2 * ref.abs().max().item() + 1e-3


def test_collective_op_nvfp4_rows_match_the_nvlink_op():
    """Both transports carry NVFP4 in one wire layout (packed e2m1 bytes; fp32 row
    scale + e4m3 block scales, padded to 16 bytes), and both quantise with the
    dispatch kernel's arithmetic (the NVLink op inside its dispatch kernel, the
    all-to-all op with kiwi_b200.ops.quant_nvfp4), so the bytes are equal."""
    from kiwi_b200.parallel.ep import KiwiEpOp
    from kiwi_b200.parallel.ep_collective import CollectiveEpOp

    kw = dict(hidden_dim=512, topk=2, num_experts_per_rank=8, max_num_inp_token_per_rank=32,
              dispatch_quant_format="fp4")
    a, b = KiwiEpOp(**kw), CollectiveEpOp(**kw)
    torch.manual_seed(4)
    x = torch.randn(32, 512, device="cuda").bfloat16()
    idx, w = moe.route_reference(torch.randn(32, 8, device="cuda"), 2)
    ra, _, sa, _, ca = a.dispatch(x, w, None, idx)
    rb, _, sb, _, cb = b.dispatch(x, w, None, idx)
    torch.cuda.synchronize()
    a.check()
    n = int(ca.item())
    assert n == int(cb.item()) == 32
    assert tuple(ra[:n].shape) == tuple(rb[:n].shape) and sa.shape[1] >= sb.shape[1]
    assert torch.equal(ra[:n].view(torch.uint8), rb[:n].view(torch.uint8))
    assert torch.equal(sa[:n, :sb.shape[1]].contiguous().view(torch.uint8), sb[:n].contiguous().view(torch.uint8))
    da = moe.dequant_nvfp4(ra[:n], sa[:n, :sb.shape[1]])
    ref = moe.quant_nvfp4_reference(x)
    assert (da != ref).float().mean().item() < 1e-2
