"""kiwi::queue ring logic on the host (no GPU): a CPU thread stands in for the
producer warp, exactly as the device writes the wire format.

Mirrors the reference's unit and chunk tests (tests/queue/test_basic.hip.cpp,
tests/queue/test_chunk_queue.hip.cpp of AMDResearch/kiwi): every message size,
wrap-around in rings of 1..4096 lines, late-chunk injection, corrupt headers,
capacity checks, host poll state.
"""
import os
import random
import struct

import pytest

from kiwi_b200 import queue as kq


def test_wire_constants():
    assert kq.LINE_BYTES == 64 and kq.CHUNK_BYTES == 16
    assert kq.MAX_MESSAGE_BYTES == 4096
    # header chunk + ceil(bytes/8) payload chunks, 4 chunks per line
    assert kq.message_chunks(0) == 1 and kq.message_lines(0) == 1
    assert kq.message_lines(8) == 1 and kq.message_lines(24) == 1
    assert kq.message_lines(25) == 2 and kq.message_lines(56) == 2
    assert kq.message_lines(4096) == 129
    assert kq.lap_tag(0, 16) == 1 and kq.lap_tag(15, 16) == 1 and kq.lap_tag(16, 16) == 2
    # 16-bit wire tags cycle through 1..65535: never 0 (a zeroed word never matches)
    assert kq.lap_tag(65534 * 16, 16) == 65535 and kq.lap_tag(65535 * 16, 16) == 1


def test_tag_cycle_wraps_in_a_tiny_ring():
    """More than 65535 laps through a one-line ring: every lap's tag differs
    from the previous lap's, across the 65535 -> 1 wrap."""
    q = kq.SPSCD2HQueue(1, host_only=True)
    w = q.host_writer()
    for i in range(140_000):
        payload = struct.pack("<Q", i * 0x9E3779B97F4A7C15 % (1 << 64))
        assert w.try_push(payload, i & 0xFFFF)
        assert q.try_pop() == (payload, i & 0xFFFF)
        assert q.try_pop() is None


@pytest.mark.parametrize("cap", [0, 3, 6, 100])
def test_capacity_must_be_power_of_two(cap):
    with pytest.raises(Exception):
        kq.SPSCD2HQueue(cap, host_only=True)


def test_every_size_roundtrip():
    q = kq.SPSCD2HQueue(256, host_only=True)
    w = q.host_writer()
    rng = random.Random(1)
    for size in list(range(0, 130)) + [255, 256, 257, 511, 512, 1000, 2048, 4095, 4096]:
        payload = bytes(rng.getrandbits(8) for _ in range(size))
        assert w.try_push(payload, size * 7 + 3)
        got = q.try_pop()
        assert got == (payload, size * 7 + 3)
        assert q.try_pop() is None


@pytest.mark.parametrize("cap", [1, 2, 4, 16, 4096])
def test_wraparound_and_backpressure(cap):
    q = kq.SPSCD2HQueue(cap, host_only=True)
    w = q.host_writer()
    rng = random.Random(cap)
    max_bytes = min(kq.MAX_MESSAGE_BYTES, (cap * 4 - 1) * 8)
    sent, received = [], []
    for i in range(3 * cap + 50):
        size = rng.randint(0, max_bytes)
        payload = os.urandom(size)
        while not w.try_push(payload, i):
            got = q.try_pop()
            assert got is not None, "full ring must hold a message"
            received.append(got)
        sent.append((payload, i))
    while True:
        got = q.try_pop()
        if got is None:
            break
        received.append(got)
    assert received == sent
    assert q.consumer_position == w.head


def test_message_larger_than_ring_rejected():
    q = kq.SPSCD2HQueue(1, host_only=True)
    w = q.host_writer()
    assert w.try_push(b"x" * 24, 0)  # 1 line
    assert q.try_pop() == (b"x" * 24, 0)
    with pytest.raises(Exception):
        w.try_push(b"x" * 25, 0)  # needs 2 lines
    with pytest.raises(Exception):
        w.try_push(b"x" * 5000, 0)


def test_late_chunk_is_not_consumed():
    """A message whose chunks are only partly visible must not be popped
    (reference: late-chunk fault injection, test_chunk_queue.hip.cpp:459-553)."""
    q = kq.SPSCD2HQueue(8, host_only=True)
    w = q.host_writer()
    payload = bytes(range(100))  # 13 payload chunks + header = 14 chunks = 4 lines
    nchunks = kq.message_chunks(100)
    total = kq.message_lines(100) * 4
    # Everything but one payload chunk
    w.write_chunks(payload, 9, 0, 5)
    w.write_chunks(payload, 9, 6, total)
    assert q.try_pop() is None
    ps = q.host_poll_state()
    assert ps.ready()  # header visible, message not complete: ready() is only a hint
    w.write_chunks(payload, 9, 5, 6)
    w.advance(kq.message_lines(100))
    assert q.try_pop() == (payload, 9)
    assert nchunks == 14


def test_header_last_publication():
    q = kq.SPSCD2HQueue(4, host_only=True)
    w = q.host_writer()
    payload = b"abcdefgh" * 3
    w.write_chunks(payload, 1, 1, 4)
    assert q.try_pop() is None
    assert not q.host_poll_state().ready()
    w.write_chunks(payload, 1, 0, 1)
    w.advance(1)
    assert q.host_poll_state().ready()
    assert q.try_pop() == (payload, 1)


def test_stale_lap_not_consumed():
    """A line holding the previous lap's tag must read as empty."""
    q = kq.SPSCD2HQueue(2, host_only=True)
    w = q.host_writer()
    for i in range(2):
        assert w.try_push(b"a" * 8, i)
    assert q.try_pop() == (b"a" * 8, 0)
    assert q.try_pop() == (b"a" * 8, 1)
    assert q.try_pop() is None  # lines still carry lap-1 tags; lap 2 expected


def test_corrupt_length_raises():
    q = kq.SPSCD2HQueue(4, host_only=True)
    tag = kq.lap_tag(0, 4)
    q.corrupt_line(0, 0, 0, tag, 100000, tag)
    with pytest.raises(Exception, match="corrupt"):
        q.try_pop()


def test_missing_padding_blocks_pop_and_credit():
    """The padding chunks of a message's last line are validated before the
    consumer advances (reference: src/queue/chunk_consumer.hpp:117-121 of
    AMDResearch/kiwi): a message whose padding has not landed is not popped and
    its line is not handed back as credit; once the padding lands it pops."""
    q = kq.SPSCD2HQueue(4, host_only=True)
    w = q.host_writer()
    w.write_chunks(b"12345678", 3, 0, 2)  # header + the one payload chunk, no padding yet
    assert q.try_pop() is None
    assert q.consumer_position == 0
    w.write_chunks(b"12345678", 3, 2, 4)  # the padding lands
    w.advance(1)
    assert q.try_pop() == (b"12345678", 3)
    assert q.consumer_position == 1
    assert q.try_pop() is None


def test_late_padding_store_cannot_reach_the_next_lap():
    """MPSC hazard: producer A's padding store is delayed while producer B
    writes the next line.  The consumer holds A (and the credit for A's line)
    until A's padding lands, so A's late store lands on A's own lap and the
    next lap's message written at that line afterwards pops intact."""
    q = kq.MPSCD2HQueue(2, host_only=True)
    w = q.host_writer()
    w.write_chunks(b"AAAAAAAA", 1, 0, 2)  # A at line 0, padding delayed
    w.advance(1)
    assert w.try_push(b"BBBBBBBB", 2)     # B at line 1, complete
    assert q.try_pop() is None           # A is held: no line goes back as credit
    assert q.consumer_position == 0
    assert not w.try_push(b"CCCCCCCC", 3)  # the ring is full until A is consumed
    # A's late padding store: it carries A's (lap 0) tag and lands on A's line
    tag0 = kq.lap_tag(0, 2)
    for chunk in (2, 3):
        q.corrupt_line(0, chunk, 0, tag0, 0, tag0)
    assert q.try_pop() == (b"AAAAAAAA", 1)
    assert q.try_pop() == (b"BBBBBBBB", 2)
    assert w.try_push(b"CCCCCCCC", 3)      # lap 1 at line 0, after A's padding landed
    assert q.try_pop() == (b"CCCCCCCC", 3)


def test_wrong_tag_in_payload_chunk_blocks_pop():
    q = kq.SPSCD2HQueue(4, host_only=True)
    w = q.host_writer()
    w.write_chunks(b"12345678", 3, 0, 4)
    q.corrupt_line(0, 1, 0, 0, 0, 0)  # the payload chunk reads as never written
    assert q.try_pop() is None
    w.write_chunks(b"12345678", 3, 1, 2)
    w.advance(1)
    assert q.try_pop() == (b"12345678", 3)


def test_h2d_spsc_host_roundtrip():
    q = kq.SPSCH2DQueue(8, host_only=True)
    r = q.host_reader()
    for i in range(40):
        p = struct.pack("<QI", i * 3, i)
        while not q.try_push(p, i):
            assert r.try_pop() is not None
        # drain in a pattern that exercises credit refresh
        if i % 3 == 0:
            while r.try_pop() is not None:
                pass
    assert q.producer_position >= 40


def test_mpmc_host_full_and_payload_limit():
    q = kq.MPMCH2DQueue(4, slot_lines=2, host_only=True)
    assert q.slot_payload_bytes == 56
    for i in range(4):
        assert q.try_push(b"z" * 56, i)
    assert not q.try_push(b"z", 9)  # no consumer acked slot 0 yet
    with pytest.raises(Exception):
        q.try_push(b"z" * 57, 0)
    with pytest.raises(Exception):
        kq.MPMCH2DQueue(4, slot_lines=9, host_only=True)


def test_handle_layout_contract():
    """The byte layout external frontends rely on (reference: HANDLE_SIZE=40 and
    field offsets, python/kiwi_triton.py:36-47); here the B200 handle is 48 bytes."""
    lay = kq.handle_layout()
    assert lay["SpscD2HHandle"] == 48
    assert lay["SpscD2HHandle.ring"] == 0
    assert lay["SpscD2HHandle.consumer_pos"] == 8
    assert lay["SpscD2HHandle.err"] == 16
    assert lay["SpscD2HHandle.head"] == 24
    assert lay["SpscD2HHandle.credit_limit"] == 32
    assert lay["SpscD2HHandle.log2cap"] == 40
    assert lay["InvokeHandle<SPSC>"] == lay["SpscD2HHandle"]
    assert lay["ErrorRecord"] == 16
