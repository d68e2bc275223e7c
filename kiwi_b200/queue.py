"""kiwi_b200.queue: GPU<->host rings (bindings of ``include/kiwi/queue``).

Wire format (``include/kiwi/queue/wire.hpp``): 64-byte lines of four 16-byte
chunks; each chunk is four 32-bit words ``{16 data bits, 16-bit lap tag}``
(8 payload bytes per chunk), because GPU 8-byte stores into host memory were
seen torn between their 4-byte words on B200 hosts while single words never
were.  Chunk 0 carries ``{metadata, length}``.  Messages are 0..4096 bytes.
"""
from ._native import load as _load

_C = _load()
_q = _C.queue

MAX_MESSAGE_BYTES = _q.MAX_MESSAGE_BYTES
LINE_BYTES = _q.LINE_BYTES
CHUNK_BYTES = _q.CHUNK_BYTES
MAX_CAPACITY_LINES = _q.MAX_CAPACITY_LINES
message_lines = _q.message_lines
message_chunks = _q.message_chunks
lap_tag = _q.lap_tag
handle_layout = _q.handle_layout

SPSCD2HQueue = _q.SPSCD2HQueue
MPSCD2HQueue = _q.MPSCD2HQueue
SPSCH2DQueue = _q.SPSCH2DQueue
MPMCH2DQueue = _q.MPMCH2DQueue
HostPollState = _q.HostPollState
RingWriter = _q.RingWriter
RingReader = _q.RingReader

__all__ = [
    "MAX_MESSAGE_BYTES", "LINE_BYTES", "CHUNK_BYTES", "MAX_CAPACITY_LINES", "message_lines",
    "message_chunks", "lap_tag", "handle_layout", "SPSCD2HQueue", "MPSCD2HQueue", "SPSCH2DQueue",
    "MPMCH2DQueue", "HostPollState", "RingWriter", "RingReader",
]
