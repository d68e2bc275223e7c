"""Property-based tests (hypothesis) of the host-side logic: any message
stream through a host-only ring arrives intact and in order across
wrap-around and tag cycles; any payload reaches its callback byte for byte;
any valid EP configuration lays out aligned, non-overlapping heap regions.
(Reference test categories: the queue basic/chunk tests, the invoke
serializer tests and the EP layout tests of AMDResearch/kiwi.)"""
import os
import struct

from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from kiwi_b200 import invoke
from kiwi_b200 import queue as kq
from kiwi_b200._native import load

SETTINGS = dict(max_examples=60, deadline=None, suppress_health_check=[HealthCheck.too_slow])


@settings(**SETTINGS)
@given(log2cap=st.integers(min_value=0, max_value=6),
       sizes=st.lists(st.integers(min_value=0, max_value=600), min_size=1, max_size=80),
       seed=st.integers(min_value=0, max_value=2**32 - 1))
def test_ring_delivers_any_stream_in_order(log2cap, sizes, seed):
    cap = 1 << log2cap
    max_bytes = min(kq.MAX_MESSAGE_BYTES, (cap * 4 - 1) * 8)
    q = kq.SPSCD2HQueue(cap, host_only=True)
    w = q.host_writer()
    sent, got = [], []
    x = seed | 1
    for i, n in enumerate(sizes):
        n = min(n, max_bytes)
        payload = bytes(((x >> (8 * (j % 8))) + j) & 0xFF for j in range(n))
        x = (x * 6364136223846793005 + 1442695040888963407) & (2**64 - 1)
        while not w.try_push(payload, i & 0xFFFF):
            r = q.try_pop()
            assert r is not None, "a full ring must hold a message"
            got.append(r)
        sent.append((payload, i & 0xFFFF))
    while (r := q.try_pop()) is not None:
        got.append(r)
    assert got == sent


@settings(**SETTINGS)
@given(payloads=st.lists(st.binary(min_size=0, max_size=512), min_size=1, max_size=40))
def test_raw_callbacks_receive_every_payload(payloads):
    ctx = invoke.Context(1, 128, host_only=True)
    seen = []
    cb = ctx.register_callback(lambda p: seen.append(bytes(p)))
    for p in payloads:
        try:
            ctx.emulate_invoke(0, cb, p)
        except Exception:
            ctx.progress(0)
            ctx.emulate_invoke(0, cb, p)
    ctx.progress(0)
    assert seen == payloads


@settings(**SETTINGS)
@given(vals=st.lists(st.tuples(st.integers(0, 2**64 - 1), st.integers(-2**31, 2**31 - 1),
                               st.floats(allow_nan=False, width=32)), min_size=1, max_size=30))
def test_typed_callbacks_unpack_packed_little_endian(vals):
    ctx = invoke.Context(1, 64, host_only=True)
    got = []
    cb = ctx.register_callback(lambda a, b, c: got.append((a, b, c)), "<Qif")
    for v in vals:
        ctx.emulate_invoke(0, cb, struct.pack("<Qif", *v))
        ctx.progress(0)
    assert got == [(a, b, struct.unpack("<f", struct.pack("<f", c))[0]) for a, b, c in vals]


@settings(**SETTINGS)
@given(world=st.sampled_from([1, 2, 4, 8, 16]), hidden_blocks=st.integers(1, 32),
       experts_per_rank=st.integers(1, 64), topk=st.integers(1, 16), max_tokens=st.integers(1, 8192),
       quant=st.sampled_from(["none", "fp8", "nvfp4"]))
def test_ep_layout_regions_aligned_and_disjoint(world, hidden_blocks, experts_per_rank, topk, max_tokens, quant):
    ep = load().ep
    experts = world * experts_per_rank
    if topk > experts:
        topk = experts
    c = ep.finalize_config(dict(world=world, rank=world - 1, hidden=512 * hidden_blocks, num_experts=experts,
                                topk=topk, max_tokens=max_tokens, quant=quant))
    slots = world * max_tokens
    hidden = 512 * hidden_blocks
    regions = [("off_flags", 2 * 16 * 128), ("off_meta", slots * c["meta_bytes"]),
               ("off_row", slots * c["row_bytes"]), ("off_scale", slots * c["scale_bytes"]),
               ("off_comb", slots * hidden * 2), ("off_combk", max_tokens * topk * hidden * 2)]
    spans = []
    for name, size in regions:
        assert c[name] % 256 == 0, name
        spans.append((c[name], c[name] + size))
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 <= b0
    assert c["heap_bytes"] >= spans[-1][1]
    assert c["meta_bytes"] % 16 == 0 and c["scale_bytes"] % 16 == 0 and c["row_bytes"] % 16 == 0
    assert c["local_per_token"] == min(topk, experts_per_rank)


def test_tag_cycle_never_zero_and_changes_every_lap():
    for lap in list(range(0, 70000, 997)) + [65533, 65534, 65535, 65536, 131070, 131071]:
        t0 = kq.lap_tag(lap * 16, 16)
        t1 = kq.lap_tag((lap + 1) * 16, 16)
        assert 1 <= t0 <= 65535 and t0 != t1


# ---- native print formatter vs Python's printf-compatible % operator ----

_INT_CODES = {"b": (-128, 127), "B": (0, 255), "h": (-(1 << 15), (1 << 15) - 1), "H": (0, (1 << 16) - 1),
              "i": (-(1 << 31), (1 << 31) - 1), "I": (0, (1 << 32) - 1), "q": (-(1 << 63), (1 << 63) - 1),
              "Q": (0, (1 << 64) - 1)}


@st.composite
def _print_case(draw):
    """(C format, the same format for Python's %, struct codes, values).  The
    generator avoids the combinations where Python's % differs from C's printf:
    the 0 flag with an integer precision, +/space with x, X, o, and a zero
    printed with precision 0."""
    fmt, py_fmt, codes, values = "", "", "", []
    for _ in range(draw(st.integers(0, 4))):
        lit = draw(st.text(alphabet="ab =:|-", max_size=4))
        width = draw(st.sampled_from(["", "3", "12"]))
        if draw(st.booleans()):
            conv = draw(st.sampled_from("dixXo"))
            code = draw(st.sampled_from("BHIQ" if conv in "xXo" else sorted(_INT_CODES)))
            lo, hi = _INT_CODES[code]
            v = draw(st.integers(lo, hi))
            prec = draw(st.sampled_from(["", ".0", ".3"])) if conv in "di" else ""
            if prec == ".0" and v == 0:  # C prints nothing here, Python's % prints 0
                prec = ""
            flag_set = "-" if conv in "xXo" else ("-+ " if prec else "-+ 0")
            if v > (1 << 63) - 1:  # printed through %u: no sign flags (documented in printer.hpp)
                flag_set = flag_set.replace("+", "").replace(" ", "")
            flags = "".join(sorted(set(draw(st.text(alphabet=flag_set, max_size=2)))))
            length = draw(st.sampled_from(["", "l", "ll", "h"]))  # replaced by the argument's own
            fmt += lit + "%" + flags + width + prec + length + conv
            py_fmt += lit + "%" + flags + width + prec + conv
        else:
            code = draw(st.sampled_from("fd"))
            v = draw(st.floats(-1e6, 1e6, allow_nan=False, width=32 if code == "f" else 64))
            conv = draw(st.sampled_from("efgEG"))
            prec = draw(st.sampled_from(["", ".0", ".3"]))
            flags = "".join(sorted(set(draw(st.text(alphabet="-+ 0", max_size=2)))))
            fmt += lit + "%" + flags + width + prec + conv
            py_fmt += lit + "%" + flags + width + prec + conv
        codes += code
        values.append(v)
    tail = draw(st.text(alphabet="xyz ", max_size=3)) + draw(st.sampled_from(["", "%%"]))
    return fmt + tail, py_fmt + tail, codes, values


@settings(max_examples=int(os.environ.get("KIWI_PROPERTY_EXAMPLES", "400")), deadline=None)
@given(_print_case())
def test_native_print_matches_printf_semantics(case):
    fmt, py_fmt, codes, values = case
    payload = struct.pack("<" + codes, *values)
    got = load().print_format.format(fmt, "<" + codes, payload)
    vals = struct.unpack("<" + codes, payload)  # float32 rounding as the device would send it
    assert got == py_fmt % tuple(vals)


_U64 = st.integers(0, (1 << 64) - 1)


@settings(max_examples=int(os.environ.get("KIWI_PROPERTY_EXAMPLES", "400")), deadline=None)
@given(st.integers(1, 16), _U64, st.integers(-2, 18), _U64, _U64)
def test_checked_mode_rule_matches_interval_model(world, limit, rank, off, nbytes):
    """The P2P checked mode admits exactly the accesses whose byte interval
    lies inside [0, limit) of an existing rank, with no wrap-around."""
    want = 0 <= rank < world and off + nbytes <= limit
    assert load().p2p.heap_range_ok(world, limit, rank, off, nbytes) == want


@settings(max_examples=int(os.environ.get("KIWI_PROPERTY_EXAMPLES", "400")), deadline=None)
@given(st.lists(st.integers(1, (1 << 63) - 1), min_size=4, max_size=64))
def test_debug_words_decode_inverts_the_device_encoding(times):
    """Start words (0 and 2 of each phase) are stored as ~t, end words as t;
    0 stays 'not recorded'."""
    mask = (1 << 64) - 1
    raw = [(~t & mask) if (i % 4) % 2 == 0 else t for i, t in enumerate(times)]
    raw[0] = 0
    got = load().ep.decode_debug_words(raw)
    assert got[0] == 0 and got[1:] == times[1:]


@settings(max_examples=int(os.environ.get("KIWI_PROPERTY_EXAMPLES", "200")), deadline=None)
@given(st.integers(0, 4), st.integers(1, 3), st.lists(st.one_of(st.binary(max_size=56), st.none()), max_size=120))
def test_mpmc_h2d_fifo_and_full_with_stand_in_consumer(log2slots, slot_lines, ops):
    """MPMC host-to-device queue against a deque model, with the CPU stand-in
    for the device consumers: bytes = push (False exactly when every slot
    holds an unconsumed message), None = pop (FIFO; None when empty)."""
    import collections

    slots = 1 << log2slots
    q = kq.MPMCH2DQueue(slots, slot_lines, host_only=True)
    payload_max = q.slot_payload_bytes
    model = collections.deque()
    for i, op in enumerate(ops):
        if op is None:
            got = q.host_try_pop()
            if model:
                assert got == model.popleft()
            else:
                assert got is None
        else:
            data = op[:payload_max]
            ok = q.try_push(data, i % 251)
            assert ok == (len(model) < slots)
            if ok:
                model.append((data, i % 251))
    while model:
        assert q.host_try_pop() == model.popleft()
    assert q.host_try_pop() is None


@settings(max_examples=40, deadline=None, suppress_health_check=[HealthCheck.too_slow])
@given(tokens=st.integers(min_value=0, max_value=24), topk=st.integers(min_value=1, max_value=4),
       epr=st.integers(min_value=1, max_value=6), seed=st.integers(min_value=0, max_value=2**31 - 1))
def test_collective_ep_op_round_trips_any_routing(tokens, topk, epr, seed):
    """World of one: any routing delivers every token once, in order, with its
    ids and weights, and combine returns it unchanged."""
    import torch

    from kiwi_b200.parallel.ep_collective import CollectiveEpOp

    topk = min(topk, epr)
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(tokens, 128, generator=g).bfloat16()
    idx = torch.stack([torch.randperm(epr, generator=g)[:topk] for _ in range(tokens)]) if tokens else \
        torch.empty(0, topk, dtype=torch.int64)
    w = torch.rand(tokens, topk, generator=g)
    op = CollectiveEpOp(hidden_dim=128, topk=topk, num_experts_per_rank=epr, max_num_inp_token_per_rank=24,
                        device="cpu")
    out, ow, _, oidx, cnt = op.dispatch(x, w, None, idx)
    assert int(cnt.item()) == tokens
    assert torch.equal(out, x) and torch.equal(oidx, idx.to(torch.int32)) and torch.equal(ow, w)
    res, _ = op.combine(out)
    assert torch.equal(res, x)


@settings(max_examples=40, deadline=None, suppress_health_check=[HealthCheck.too_slow])
@given(counts=st.lists(st.integers(min_value=0, max_value=9), min_size=1, max_size=5), swiglu=st.booleans(),
       seed=st.integers(min_value=0, max_value=2**31 - 1))
def test_grouped_gemm_reference_is_a_per_group_matmul(counts, swiglu, seed):
    import torch

    from kiwi_b200.ops import grouped_gemm_reference

    g = torch.Generator().manual_seed(seed)
    rows, n, k = sum(counts), 256, 32
    a = torch.randn(rows, k, generator=g)
    b = torch.randn(len(counts) * n, k, generator=g)
    got = grouped_gemm_reference(a, b, counts, swiglu)
    off = 0
    for e, c in enumerate(counts):
        y = a[off:off + c] @ b[e * n:(e + 1) * n].t()
        if swiglu:
            y = torch.nn.functional.silu(y[:, :128]) * y[:, 128:]
        assert torch.allclose(got[off:off + c], y, rtol=1e-5, atol=1e-4)
        off += c
    assert got.shape[0] == rows
