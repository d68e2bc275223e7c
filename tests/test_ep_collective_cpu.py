"""CollectiveEpOp: KiwiEpOp's dispatch / combine contract over all-to-all,
checked on CPU (world of 1 in-process, two gloo ranks as processes) against
the contract computed directly from every rank's inputs."""
import multiprocessing as mp
import os
import socket

import pytest
import torch

from kiwi_b200.models import moe
from kiwi_b200.parallel.ep_collective import CollectiveEpOp

HIDDEN, TOPK, EPR, TOKENS = 256, 3, 4, 24


def inputs(rank, world, tokens=TOKENS):
    """Seeded per-rank inputs every process can regenerate."""
    g = torch.Generator().manual_seed(100 + rank)
    x = torch.randn(tokens, HIDDEN, generator=g).bfloat16()
    logits = torch.randn(tokens, EPR * world, generator=g)
    idx, w = moe.route_reference(logits, TOPK)
    return x, idx.to(torch.int32), w.float()


def expected(rank, world, quant):
    """(rows, weights, indices, positions) rank `rank` must receive, in (source, token) order."""
    rows, ws, ids, pos = [], [], [], []
    for s in range(world):
        x, idx, w = inputs(s, world)
        for t in range(x.shape[0]):
            if bool(((idx[t].long() // EPR) == rank).any()):
                rows.append(x[t])
                ws.append(w[t])
                ids.append(idx[t])
                pos.append(s * world * TOKENS + t)
    rows = torch.stack(rows) if rows else torch.empty(0, HIDDEN, dtype=torch.bfloat16)
    return rows, torch.stack(ws), torch.stack(ids), pos


def check_rank(op, rank, world, quant):
    x, idx, w = inputs(rank, world)
    out, ow, sc, oidx, cnt = op.dispatch(x, w, None, idx)
    rows, ws, ids, pos = expected(rank, world, quant)
    n = int(cnt.item())
    assert n == rows.shape[0]
    assert torch.equal(oidx[:n], ids) and torch.equal(ow[:n], ws)
    assert op.get_dispatch_src_token_pos().tolist() == pos
    assert [op.decode_send_flat_idx(p) for p in pos] == [(p // (world * TOKENS), p % (world * TOKENS)) for p in pos]
    if quant == "fp8":
        codes, scales = moe.quant_fp8_codes(rows)
        assert out.dtype == torch.float8_e4m3fn
        assert torch.equal(out[:n].view(torch.uint8), codes.view(torch.uint8)) and torch.equal(sc[:n], scales)
        back = moe.quant_fp8_reference(rows).bfloat16()
    elif quant == "fp4":
        codes, scales = moe.quant_nvfp4_codes(rows)
        assert out.dtype == torch.uint8 and tuple(out.shape[1:]) == (HIDDEN // 2,)
        assert torch.equal(out[:n], codes) and torch.equal(sc[:n], scales)
        back = moe.dequant_nvfp4(out[:n], sc[:n]).bfloat16()
    else:
        assert sc is None and torch.equal(out[:n], rows)
        back = out[:n].clone()
    # combine: every destination returns the token's (dequantised) row; the source sums them
    res, _ = op.combine(back, None, oidx)
    dests = (idx.long() // EPR)
    want = torch.zeros(x.shape[0], HIDDEN)
    ref_rows = {"fp8": moe.quant_fp8_reference, "fp4": moe.quant_nvfp4_reference}.get(quant, lambda v: v.float())(x)
    for t in range(x.shape[0]):
        k = len(set(dests[t].tolist()))
        want[t] = ref_rows[t].bfloat16().float() * k
    assert (res.float() - want).abs().max().item() <= 2e-2 * want.abs().max().item() + 1e-3


@pytest.mark.parametrize("quant", ["none", "fp8", "fp4"])
def test_world_of_one(quant):
    op = CollectiveEpOp(hidden_dim=HIDDEN, topk=TOPK, num_experts_per_rank=EPR, max_num_inp_token_per_rank=TOKENS,
                        dispatch_quant_format=quant, device="cpu")
    for _ in range(2):  # rounds are independent
        check_rank(op, 0, 1, quant)


def _member(rank, port, quant, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                      LOCAL_RANK=str(rank))
    try:
        from kiwi_b200.utils import dist as kdist

        kdist.init(backend="gloo", timeout_s=30.0, device=False)
        op = CollectiveEpOp(hidden_dim=HIDDEN, topk=TOPK, num_experts_per_rank=EPR,
                            max_num_inp_token_per_rank=TOKENS, dispatch_quant_format=quant, device="cpu")
        for _ in range(2):
            check_rank(op, rank, 2, quant)
        kdist.dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        import traceback

        q.put((rank, f"{type(e).__name__}: {e}\n{traceback.format_exc()[-2000:]}"))


@pytest.mark.parametrize("quant", ["none", "fp8", "fp4"])
def test_two_gloo_ranks(quant):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_member, args=(r, port, quant, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=180) for _ in ps)
    for p in ps:
        p.join(timeout=30)
    assert got == {0: "ok", 1: "ok"}, got


def test_float32_combine_sums_exactly():
    op = CollectiveEpOp(hidden_dim=HIDDEN, topk=TOPK, num_experts_per_rank=EPR, max_num_inp_token_per_rank=TOKENS,
                        combine_dtype=torch.float32, device="cpu")
    x, idx, w = inputs(0, 1)
    out, _, _, _, cnt = op.dispatch(x, w, None, idx)
    n = int(cnt.item())
    rows = torch.randn(n, HIDDEN)  # fp32 expert outputs, one per received row
    res, _ = op.combine(rows)
    assert res.dtype == torch.float32 and torch.equal(res, rows)  # world of 1: one row per token


def test_prequantised_fp8_input_travels_unchanged():
    op = CollectiveEpOp(hidden_dim=HIDDEN, topk=TOPK, num_experts_per_rank=EPR, max_num_inp_token_per_rank=TOKENS,
                        dispatch_quant_format="fp8", device="cpu")
    x, idx, w = inputs(0, 1)
    codes = (torch.randn(TOKENS, HIDDEN) * 50).to(torch.float8_e4m3fn)
    scales = torch.rand(TOKENS, 4) + 0.1  # the caller's own scale layout (4 per row here)
    out, _, sc, _, cnt = op.dispatch(codes, w, scales, idx)
    n = int(cnt.item())
    assert torch.equal(out[:n].view(torch.uint8), codes.view(torch.uint8)) and torch.equal(sc[:n], scales)
    with pytest.raises(ValueError):
        op.dispatch(codes, w, None, idx)
    bf16_op = CollectiveEpOp(hidden_dim=HIDDEN, topk=TOPK, num_experts_per_rank=EPR,
                             max_num_inp_token_per_rank=TOKENS, device="cpu")
    with pytest.raises(ValueError):
        bf16_op.dispatch(codes, w, scales, idx)


def test_registered_combine_buffer():
    op = CollectiveEpOp(hidden_dim=HIDDEN, topk=TOPK, num_experts_per_rank=EPR, max_num_inp_token_per_rank=TOKENS,
                        device="cpu")
    buf = op.get_registered_combine_input_buffer(torch.bfloat16)
    assert tuple(buf.shape) == (TOKENS, HIDDEN) and buf is op.get_registered_combine_input_buffer()
    x, idx, w = inputs(0, 1)
    out, _, _, _, cnt = op.dispatch(x, w, None, idx)
    n = int(cnt.item())
    buf[:n].copy_(out[:n])
    res, _ = op.combine(buf)
    assert torch.equal(res, x)
    with pytest.raises(ValueError):
        op.get_registered_combine_input_buffer(torch.float32)


def test_constructor_checks():
    with pytest.raises(TypeError):
        CollectiveEpOp(0, 1, 256)
    with pytest.raises(ValueError):
        CollectiveEpOp(hidden_dim=256, topk=2, num_experts_per_rank=4, max_num_inp_token_per_rank=8,
                       combine_dtype=torch.float16, device="cpu")
    with pytest.raises(ValueError):
        CollectiveEpOp(hidden_dim=256, topk=2, num_experts_per_rank=4, max_num_inp_token_per_rank=8,
                       dispatch_quant_format="int4", device="cpu")
    with pytest.raises(ValueError):
        CollectiveEpOp(hidden_dim=200, topk=2, num_experts_per_rank=4, max_num_inp_token_per_rank=8,
                       dispatch_quant_format="fp4", device="cpu")
    with pytest.raises(ValueError):
        CollectiveEpOp(hidden_dim=200, topk=2, num_experts_per_rank=4, max_num_inp_token_per_rank=8,
                       dispatch_quant_format="fp8", device="cpu")
    op = CollectiveEpOp(hidden_dim=256, topk=2, num_experts_per_rank=4, max_num_inp_token_per_rank=8, device="cpu")
    with pytest.raises(RuntimeError):
        op.combine(torch.zeros(1, 256).bfloat16())


# -- CollectiveMoE: the whole layer over the all-to-all transport ---------------------------------

def _moe_cfg(world, quant):
    return moe.MoEConfig(hidden=256, ffn=128, num_experts=3 * world, topk=2, tokens_per_rank=20, quant=quant,
                         name="t")


def check_moe(rank, world, quant):
    from kiwi_b200.parallel.ep_collective import CollectiveMoE

    cfg = _moe_cfg(world, quant)
    layer = CollectiveMoE(cfg, device="cpu")
    for step in range(2):
        x, logits = moe.synthetic_inputs(cfg, rank, "cpu", tokens=20 - 6 * step, step=step)
        out = layer(x, logits)
        idx, w = moe.route_reference(logits, cfg.topk)
        ref = moe.moe_reference(cfg, x, idx, w, device="cpu")
        err = (out.float() - ref).abs().max().item()
        assert out.shape == ref.shape and err <= 2e-2 * ref.abs().max().item() + 1e-3, (rank, step, err)


@pytest.mark.parametrize("quant", ["none", "fp8", "nvfp4"])
def test_moe_layer_world_of_one(quant):
    check_moe(0, 1, quant)


def _moe_member(rank, port, quant, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                      LOCAL_RANK=str(rank))
    try:
        from kiwi_b200.utils import dist as kdist

        kdist.init(backend="gloo", timeout_s=30.0, device=False)
        check_moe(rank, 2, quant)
        kdist.dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        import traceback

        q.put((rank, f"{type(e).__name__}: {e}\n{traceback.format_exc()[-2000:]}"))


def test_moe_layer_two_gloo_ranks():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_moe_member, args=(r, port, "fp8", q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=180) for _ in ps)
    for p in ps:
        p.join(timeout=30)
    assert got == {0: "ok", 1: "ok"}, got


def test_moe_layer_rejects_unknown_wire_formats():
    from kiwi_b200.parallel.ep_collective import CollectiveMoE

    with pytest.raises(ValueError):
        CollectiveMoE(_moe_cfg(1, "int8"), device="cpu")


def test_token_sweep_including_zero():
    """Rounds of 0 to max tokens in a row on one op (world of one)."""
    op = CollectiveEpOp(hidden_dim=HIDDEN, topk=TOPK, num_experts_per_rank=EPR, max_num_inp_token_per_rank=TOKENS,
                        device="cpu")
    for t in (0, 1, 2, 13, TOKENS, 0, 5):
        x, idx, w = inputs(t, 1, tokens=t)
        out, ow, _, oidx, cnt = op.dispatch(x, w, None, idx)
        assert int(cnt.item()) == t and torch.equal(out, x) and torch.equal(oidx, idx)
        assert op.get_dispatch_src_token_pos().tolist() == list(range(t))
        res, _ = op.combine(out)
        assert res.shape == (t, HIDDEN) and torch.equal(res, x)
    x, idx, w = inputs(0, 1, tokens=TOKENS + 1)
    with pytest.raises(ValueError):
        op.dispatch(x, w, None, idx)  # more than max_num_inp_token_per_rank


def _uneven_member(rank, port, q):
    """Rank 0 has no tokens; rank 1 routes every token to its own experts."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                      LOCAL_RANK=str(rank))
    try:
        from kiwi_b200.utils import dist as kdist

        kdist.init(backend="gloo", timeout_s=30.0, device=False)
        op = CollectiveEpOp(hidden_dim=HIDDEN, topk=TOPK, num_experts_per_rank=EPR,
                            max_num_inp_token_per_rank=TOKENS, device="cpu")
        t = 0 if rank == 0 else 9
        x = torch.randn(t, HIDDEN).bfloat16()
        idx = (EPR + torch.arange(t * TOPK) % EPR).view(t, TOPK).to(torch.int32)
        w = torch.full((t, TOPK), 1.0 / TOPK)
        out, _, _, _, cnt = op.dispatch(x, w, None, idx)
        assert int(cnt.item()) == (0 if rank == 0 else 9)
        res, _ = op.combine(out)
        assert res.shape == (t, HIDDEN) and torch.equal(res, x)
        kdist.dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        import traceback

        q.put((rank, f"{type(e).__name__}: {e}\n{traceback.format_exc()[-2000:]}"))


def test_two_gloo_ranks_with_empty_sends():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_uneven_member, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=180) for _ in ps)
    for p in ps:
        p.join(timeout=30)
    assert got == {0: "ok", 1: "ok"}, got


def test_out_of_range_expert_ids_are_rejected():
    op = CollectiveEpOp(hidden_dim=HIDDEN, topk=TOPK, num_experts_per_rank=EPR, max_num_inp_token_per_rank=TOKENS,
                        device="cpu")
    x, idx, w = inputs(0, 1)
    for bad in (EPR, -1):
        idx2 = idx.clone()
        idx2[3, 1] = bad
        with pytest.raises(ValueError):
            op.dispatch(x, w, None, idx2)


def test_fp8_combine_sums_codes_and_saturates():
    op = CollectiveEpOp(hidden_dim=HIDDEN, topk=TOPK, num_experts_per_rank=EPR, max_num_inp_token_per_rank=TOKENS,
                        combine_dtype=torch.float8_e4m3fn, device="cpu")
    x, idx, w = inputs(0, 1)
    _, _, _, _, cnt = op.dispatch(x, w, None, idx)
    n = int(cnt.item())
    rows = (torch.randn(n, HIDDEN) * 30).to(torch.float8_e4m3fn)
    rows[0, 0] = torch.tensor(-0.0).to(torch.float8_e4m3fn)  # always exercise the -0 code
    res, _ = op.combine(rows)
    assert res.dtype == torch.float8_e4m3fn
    # one row per token at world 1: the same values (a -0 code comes back as +0 after the fp32 sum)
    assert torch.equal(res.float(), rows.float())
    big = torch.full((n, HIDDEN), 1000.0)  # bf16 / fp32 rows past the FP8 range saturate, never NaN
    res, _ = op.combine(big)
    assert (res.float() == 448.0).all()
    buf = op.get_registered_combine_input_buffer()
    assert buf.dtype == torch.float8_e4m3fn


def test_fp4_codes_round_trip_and_pack_low_nibble_first():
    vals = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.5, -6.0, 7.0, -100.0, 0.74, 0.76, 2.5, 5.0])
    codes = moe.fp4_codes(vals)
    back = moe.fp4_unpack(moe.fp4_pack(codes))
    want = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.5, -6.0, 6.0, -6.0, 0.5, 1.0, 2.0, 4.0])
    assert torch.equal(back, want)  # 0.75 -> 0.5 / 1.0 by distance; ties 2.5 -> 2, 5 -> 4 (even mantissa)
    assert int(moe.fp4_pack(moe.fp4_codes(torch.tensor([1.0, -2.0])))[0]) == 0x2 | (0xC << 4)


def test_fp4_combine_sums_and_requantises():
    op = CollectiveEpOp(hidden_dim=HIDDEN, topk=TOPK, num_experts_per_rank=EPR, max_num_inp_token_per_rank=TOKENS,
                        combine_dtype=torch.float4_e2m1fn_x2, device="cpu")
    x, idx, w = inputs(0, 1)
    _, _, _, _, cnt = op.dispatch(x, w, None, idx)
    n = int(cnt.item())
    vals = moe.FP4_VALUES[torch.randint(0, 8, (n, HIDDEN))] * torch.where(torch.rand(n, HIDDEN) < 0.5, -1.0, 1.0)
    packed = moe.fp4_pack(moe.fp4_codes(vals)).view(torch.float4_e2m1fn_x2)
    res, _ = op.combine(packed)
    assert res.dtype == torch.float4_e2m1fn_x2 and tuple(res.shape) == (TOKENS, HIDDEN // 2)
    assert torch.equal(moe.fp4_unpack(res), vals)  # world of one: one row per token
    res, _ = op.combine(torch.full((n, HIDDEN), 9.0))  # float rows are quantised, saturating at 6
    assert (moe.fp4_unpack(res) == 6.0).all()
    assert tuple(op.get_registered_combine_input_buffer().shape) == (TOKENS * 1, HIDDEN // 2)
    with pytest.raises(ValueError):
        CollectiveEpOp(hidden_dim=255, topk=1, num_experts_per_rank=1, max_num_inp_token_per_rank=1,
                       combine_dtype=torch.float4_e2m1fn_x2, device="cpu")


def test_prequantised_fp4_input_travels_unchanged():
    op = CollectiveEpOp(hidden_dim=HIDDEN, topk=TOPK, num_experts_per_rank=EPR, max_num_inp_token_per_rank=TOKENS,
                        dispatch_quant_format="fp4", device="cpu")
    x, idx, w = inputs(0, 1)
    codes = torch.randint(0, 256, (TOKENS, HIDDEN // 2), dtype=torch.uint8)
    scales = torch.rand(TOKENS, 5)  # the caller's own layout: 20 bytes per token
    out, _, sc, _, cnt = op.dispatch(codes.view(torch.float4_e2m1fn_x2), w, scales, idx)
    n = int(cnt.item())
    assert torch.equal(out[:n], codes) and torch.equal(sc[:n], scales.view(torch.uint8))
    with pytest.raises(ValueError):
        op.dispatch(codes, w, None, idx)
