"""EP configuration, heap layout and the fp32 reference model (CPU).

Mirrors the reference's layout unit tests (apps/ep/tests/test_rcomp_readiness_layout.hip.cpp,
test_ep_block_count.hip.cpp of AMDResearch/kiwi): capacities, alignment and
non-overlap of every heap region for world sizes 1..16.
"""
import pytest
import torch

import kiwi_b200
from kiwi_b200.models import moe

C = kiwi_b200.native()


def cfg(**kw):
    d = dict(world=8, rank=3, hidden=7168, num_experts=256, topk=8, max_tokens=4096, quant="fp8")
    d.update(kw)
    return C.ep.finalize_config(d)


def test_fp8_layout_of_the_benchmark_config():
    c = cfg()
    assert c["experts_per_rank"] == 32
    assert c["row_bytes"] == 7168 and c["scale_bytes"] == 7168 // 128 * 4
    assert c["meta_bytes"] == 16 + 8 * 8
    slots = 8 * 4096
    regions = [("off_flags", 2 * 16 * 128), ("off_meta", slots * c["meta_bytes"]),
               ("off_row", slots * c["row_bytes"]), ("off_scale", slots * c["scale_bytes"]),
               ("off_comb", slots * 7168 * 2), ("off_combk", 4096 * 8 * 7168 * 2)]
    ends = []
    for name, size in regions:
        assert c[name] % 256 == 0, name
        ends.append((c[name], c[name] + size))
    for (a0, a1), (b0, b1) in zip(ends, ends[1:]):
        assert a1 <= b0
    assert c["heap_bytes"] >= ends[-1][1]
    assert c["max_pairs"] == 8 * 4096 * 8
    assert c["local_per_token"] == 8


@pytest.mark.parametrize("world", [1, 2, 4, 8, 16])
@pytest.mark.parametrize("quant", ["fp8", "nvfp4", "none"])
def test_layout_alignment(world, quant):
    c = cfg(world=world, rank=world - 1, num_experts=256 if world <= 16 else 256, quant=quant)
    for k in ("off_meta", "off_row", "off_scale", "off_comb", "off_combk"):
        assert c[k] % 256 == 0
    assert c["row_bytes"] % 16 == 0 and c["scale_bytes"] % 16 == 0 and c["meta_bytes"] % 16 == 0
    if quant == "nvfp4":
        assert c["row_bytes"] == 7168 // 2
        assert c["scale_bytes"] >= 7168 // 16 + 4


@pytest.mark.parametrize("bad", [dict(world=0), dict(rank=8), dict(num_experts=100), dict(topk=17),
                                 dict(topk=0), dict(hidden=1000), dict(quant="int3"), dict(max_tokens=0)])
def test_config_rejects(bad):
    with pytest.raises(Exception):
        cfg(**bad)


def test_interleave_gate_up_layout():
    w1 = torch.arange(512 * 4, dtype=torch.float32).view(512, 4)
    w3 = -w1
    w13 = moe.interleave_gate_up(w1, w3)
    assert w13.shape == (1024, 4)
    for t in range(4):
        assert torch.equal(w13[256 * t:256 * t + 128], w1[128 * t:128 * t + 128])
        assert torch.equal(w13[256 * t + 128:256 * t + 256], w3[128 * t:128 * t + 128])


def test_route_reference_softmax_over_topk():
    logits = torch.randn(50, 64)
    idx, w = moe.route_reference(logits, 6)
    assert idx.shape == (50, 6) and torch.allclose(w.sum(-1), torch.ones(50))
    v, _ = torch.topk(logits, 6)
    assert torch.equal(idx.long(), torch.topk(logits, 6).indices)
    assert (w[:, :-1] >= w[:, 1:]).all()


def test_fp8_reference_error_bound():
    x = torch.randn(64, 1024)
    xq = moe.quant_fp8_reference(x)
    # e4m3 has 3 mantissa bits: relative error <= 2^-4 of each block's amax scale
    blocks = x.view(64, 8, 128)
    err = (xq - x).view(64, 8, 128).abs()
    bound = blocks.abs().amax(-1, keepdim=True) / 448 * 32 / 2 + 1e-6  # half ulp at the top binade
    assert (err <= bound).all()


def test_nvfp4_reference_grid_and_error():
    x = torch.randn(16, 512)
    xq = moe.quant_nvfp4_reference(x)
    rel = ((xq - x).abs().sum() / x.abs().sum()).item()
    assert rel < 0.15
    assert torch.equal(moe.quant_nvfp4_reference(torch.zeros(2, 512)), torch.zeros(2, 512))


def test_reference_layer_is_linear_in_routing_weight():
    c = moe.MoEConfig(hidden=256, ffn=128, num_experts=8, topk=2, tokens_per_rank=5, quant="none")
    x, logits = moe.synthetic_inputs(c, 0, "cpu")
    idx, w = moe.route_reference(logits, 2)
    y1 = moe.moe_reference(c, x, idx, w, device="cpu")
    y2 = moe.moe_reference(c, x, idx, 2 * w, device="cpu")
    assert torch.allclose(2 * y1, y2, rtol=1e-4, atol=1e-5)


def test_weights_depend_only_on_global_expert_id():
    c = moe.MoEConfig(hidden=256, ffn=128, num_experts=8, topk=2)
    w13_1, w2_1 = moe.local_expert_weights(c, 0, 1, "cpu")
    w13_2, w2_2 = moe.local_expert_weights(c, 1, 2, "cpu")
    e_local = 4
    assert torch.equal(w13_1[e_local * 256:], w13_2)
    assert torch.equal(w2_1[e_local * 256:], w2_2)


def test_zipf_skews_routing():
    c = moe.CONFIGS["nvfp4"]
    small = moe.MoEConfig(hidden=512, ffn=256, num_experts=64, topk=6, tokens_per_rank=4096, zipf=1.2)
    _, logits = moe.synthetic_inputs(small, 0, "cpu")
    idx, _ = moe.route_reference(logits, 6)
    counts = torch.bincount(idx.flatten().long(), minlength=64).float()
    assert counts.max() / counts.mean() > 3.0
    assert c.quant == "nvfp4" and c.topk == 6


def test_tuning_table_and_overrides():
    """B200 tuning table (reference: apps/ep/ep_tuning.hpp runtime tables):
    latency vs throughput entries, and KIWI_EP_TUNING overrides."""
    from kiwi_b200._native import load

    ep = load().ep
    cfg = dict(world=8, rank=0, hidden=7168, num_experts=256, topk=8, max_tokens=4096, quant="fp8")
    t = ep.tune(cfg, 148, "")
    assert t["fused_combine"] and not t["gather_a"] and not t["gemm_pair"] and t["gemm_pair_auto"] and not t["gemm_split"]
    assert not t["gemm2_pair"] and t["gemm_m64_tails"]
    assert t["recv_blocks"] == 8 * 148 and t["combine_blocks"] == 8 * 148 and t["dispatch_blocks"] == 0
    assert "throughput" in t["source"]
    lat = ep.tune({**cfg, "max_tokens": 128}, 148, "")
    assert lat["recv_blocks"] == 4 * 148 and "latency" in lat["source"]
    o = ep.tune(cfg, 148, "gather_a=1,dispatch_blocks=296,fused_combine=off")
    assert o["gather_a"] and o["dispatch_blocks"] == 296 and not o["fused_combine"]
    assert o["source"].endswith("KIWI_EP_TUNING")
    assert ep.tune(cfg, 148, "gemm2_pair=1")["gemm2_pair"]
    assert not ep.tune(cfg, 148, "gemm_m64_tails=0")["gemm_m64_tails"]
    for bad in ("nope=1", "gather_a=maybe", "recv_blocks=0", "dispatch_blocks", "dispatch_blocks=12abc",
                "recv_blocks=99999999999", "combine_blocks=2000000", "dispatch_blocks=-1", "recv_blocks= 5"):
        with pytest.raises(Exception):
            ep.tune(cfg, 148, bad)
    assert ep.tune(cfg, 148, "recv_blocks=1048576,,combine_blocks=1")["recv_blocks"] == 1 << 20


# ---- device phase timing: layout and decoding (the kernels' side is a GPU test) ----

def test_debug_timing_layout_and_names():
    names = list(C.ep.DEBUG_PHASES)
    assert names[:3] == ["route", "begin", "dispatch"]
    for n in ("recv_count", "recv_assign", "recv_copy", "gemm1", "gemm2", "combine_send", "combine_recv",
              "recv_compact", "gather_rows", "combine_rows"):
        assert n in names
    assert len(set(names)) == len(names)
    assert C.ep.DEBUG_WORDS_PER_PHASE == 4
    assert C.ep.DEBUG_TIME_WORDS >= 4 * len(names)
    assert list(C.ep.DEBUG_META)[:3] == ["rank", "world", "tokens"]


def test_debug_words_decode_start_slots_from_complement():
    mask = (1 << 64) - 1
    raw = [~1000 & mask, 2500, ~1200 & mask, 2000, 0, 0, 0, 0, ~3000 & mask, 3400, 0, 0]
    assert C.ep.decode_debug_words(raw) == [1000, 2500, 1200, 2000, 0, 0, 0, 0, 3000, 3400, 0, 0]


def test_debug_phases_table_relative_to_first_stamp():
    from kiwi_b200.parallel.ep import debug_phases, format_debug_timing

    names = list(C.ep.DEBUG_PHASES)
    ticks = [0] * C.ep.DEBUG_TIME_WORDS
    d, rc = names.index("dispatch"), names.index("recv_count")
    ticks[4 * d:4 * d + 2] = [10_000, 14_000]
    ticks[4 * rc:4 * rc + 4] = [14_500, 30_000, 14_600, 29_000]
    snap = {"time_ticks": ticks, "phase_names": names, "meta": [3, 8, 128] + [0] * 29,
            "meta_names": list(C.ep.DEBUG_META)}
    ph = debug_phases(snap)
    assert set(ph) == {"dispatch", "recv_count"}
    assert ph["dispatch"] == {"start_us": 0.0, "end_us": 4.0, "us": 4.0}
    assert ph["recv_count"]["start_us"] == 4.5 and ph["recv_count"]["us"] == 15.5
    assert ph["recv_count"]["wait_us"] == 14.4
    text = format_debug_timing(snap)
    assert "rank=3" in text and "tokens=128" in text
    assert text.index("dispatch") < text.index("recv_count")


def test_kiwi_ep_op_source_position_encoding_round_trips():
    """get_dispatch_src_token_pos uses the reference's encoding
    src_rank * (world * max_tokens) + token, and decode_send_flat_idx inverts it."""
    from kiwi_b200.parallel.ep import KiwiEpOp, _to_send_flat_idx

    world, max_tokens = 4, 10
    slots = torch.arange(world * max_tokens)  # receive-slot order: src_rank * max_tokens + token
    enc = _to_send_flat_idx(slots, max_tokens, world)
    op = KiwiEpOp.__new__(KiwiEpOp)
    op.world_size, op.max_tokens, op.hidden_dim = world, max_tokens, 64
    op._combine_dtype, op._comb = torch.bfloat16, "bf16"
    assert op.max_num_tokens_to_send() == 40 and op.max_num_tokens_to_recv_per_rank() == 10
    for s, e in zip(slots.tolist(), enc.tolist()):
        assert op.decode_send_flat_idx(e) == (s // max_tokens, s % max_tokens)
    with pytest.raises(ValueError):
        op.get_registered_combine_input_buffer(torch.float32)
    with pytest.raises(ValueError):
        op.get_registered_combine_input_buffer(torch.bfloat16, hidden_dim=32)


def test_kiwi_ep_ext_module_surface():
    """The reference extension's module-level API under its own name."""
    from kiwi_b200.parallel import kiwi_ep_ext as ext

    assert ext.get_rank() == 0 and ext.get_nranks() == 1
    ext.barrier()
    assert ext.get_hca_name_for_gpu(0) == "" and ext.get_hca_name_for_current_gpu() == ""
    d = ext.recommended_runtime_defaults(128, 8)
    assert d["num_blocks"] > 0 and d["rcomp_backend"] == "nvlink"
    assert ext.recommended_num_blocks(4096, 8) >= ext.recommended_num_blocks(8, 8) > 0
    with ext.LciContext("") as ctx:
        assert ctx.nranks == 1
    with pytest.raises(TypeError):
        ext.KiwiEpOp(0, 1, 512)  # topk, experts per rank and max tokens missing
    with pytest.raises(ValueError):
        ext.KiwiEpOp(0, 1, 512, 2, 8, 16, torch.bfloat16, torch.bfloat16, dispatch_quant_format="int4")


@pytest.mark.parametrize("kwargs", [
    dict(combine_dtype=torch.int32),                                    # no such combine dtype
    dict(combine_dtype=torch.uint8),                                    # one-byte combine needs a quant format
    dict(combine_scale_dim=4, combine_scale_type_size=4),               # combine scales are not carried
    dict(rcomp_backend="rdma-only"),                                    # no RDMA path
    dict(dispatch_quant_format="fp8", dispatch_elem_size=2),            # FP8 wire bytes are one byte each
    dict(dispatch_dtype=torch.float16),                                 # no fp16 wire format
])
def test_kiwi_ep_op_rejects_what_it_cannot_honour(kwargs):
    """Arguments the NVLink op cannot honour raise ValueError before any device
    work (the reference raises on the same combinations or has no B200 meaning)."""
    from kiwi_b200.parallel.ep import KiwiEpOp

    base = dict(device_id=None, world_size=None, hidden_dim=512, topk=2, num_experts_per_rank=8,
                max_num_inp_token_per_rank=16)
    with pytest.raises(ValueError):
        KiwiEpOp(**{**base, **kwargs})


def test_kiwi_ep_op_rejects_unknown_arguments():
    """Keyword arguments that are not the reference's raise TypeError instead of
    being dropped."""
    from kiwi_b200.parallel.ep import KiwiEpOp

    with pytest.raises(TypeError):
        KiwiEpOp(hidden_dim=512, topk=2, num_experts_per_rank=8, max_num_inp_token_per_rank=16, use_fast_path=True)
