"""Device timing helpers: CUDA events on the launching stream, L2 flush."""
import torch


class EventTimer:
    """CUDA-event timer of a region on the current stream:
    ``with EventTimer() as t: ...`` then ``t.ms()`` after a synchronize."""
    def __init__(self):
        self.start = torch.cuda.Event(enable_timing=True)
        self.end = torch.cuda.Event(enable_timing=True)

    def __enter__(self):
        self.start.record()
        return self

    def __exit__(self, *exc):
        self.end.record()
        return False

    def ms(self):
        self.end.synchronize()
        return self.start.elapsed_time(self.end)


_flush_buf = None


def flush_l2(nbytes=256 << 20):
    """Writes a buffer larger than the 126 MB L2 so the next kernel starts cold."""
    global _flush_buf
    if _flush_buf is None or _flush_buf.numel() * 4 < nbytes:
        _flush_buf = torch.empty(nbytes // 4, dtype=torch.int32, device="cuda")
    _flush_buf.zero_()
