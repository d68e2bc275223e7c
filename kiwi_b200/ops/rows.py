"""Row copies of EP dispatch and combine as stand-alone ops: gather (pack),
scatter (unpack), plain copy, and the top-k accumulate.

CUDA tensors run the native kernels (``kiwi_b200._C.ops.rows_copy`` /
``rows_accumulate``: one CTA per row at a time, 16-byte accesses); CPU tensors
run :func:`copy_rows_reference` / :func:`accumulate_rows_reference`.  Indices
are int32; a negative index means "no row" and is skipped.  An index past the
end of its tensor is not written: the kernel sets a bit of ``error`` (1: a
source index, 2: a destination index), which :func:`check_error` turns into an
exception.  Counterparts of the reference's pack / unpack / accumulate copy
kernels (apps/ep/benchmarks/bench_ep_hidden_copy.hip.cpp of AMDResearch/kiwi).
"""
import torch

SRC_RANGE, DST_RANGE = 1, 2


def _as_index(idx, device):
    if idx is None:
        return None
    idx = torch.as_tensor(idx)
    return idx.to(device=device, dtype=torch.int32).contiguous()


def copy_rows_reference(src, dst, src_index=None, dst_index=None, rows=None):
    """CPU restatement of the copy; returns the error bits it would set."""
    n = rows if rows is not None else (len(src_index) if src_index is not None else
                                       len(dst_index) if dst_index is not None else min(len(src), len(dst)))
    err = 0
    for i in range(n):
        s = int(src_index[i]) if src_index is not None else i
        d = int(dst_index[i]) if dst_index is not None else i
        if s < 0 or d < 0:
            continue
        if s >= src.shape[0] or d >= dst.shape[0]:
            err |= (SRC_RANGE if s >= src.shape[0] else 0) | (DST_RANGE if d >= dst.shape[0] else 0)
            continue
        dst[d] = src[s]
    return err


def accumulate_rows_reference(src, index, out):
    """CPU restatement of the accumulate (fp32 sums, bf16 out); returns the error bits."""
    err = 0
    for t in range(index.shape[0]):
        acc = torch.zeros(src.shape[1], dtype=torch.float32)
        for r in index[t].tolist():
            if r < 0:
                continue
            if r >= src.shape[0]:
                err |= SRC_RANGE
                continue
            acc += src[r].float()
        out[t] = acc.to(out.dtype)
    return err


def copy_rows(src, dst, src_index=None, dst_index=None, rows=None, error=None):
    """dst[dst_index[i]] = src[src_index[i]] for i < rows (identity where an index
    is None).  Returns the error word (an int32[1] device tensor on CUDA, an int
    on CPU); nothing synchronises."""
    if not src.is_cuda:
        return copy_rows_reference(src, dst, src_index, dst_index, rows)
    from .. import native

    if error is None:
        error = torch.zeros(1, dtype=torch.int32, device=src.device)
    native().ops.rows_copy(src, dst, _as_index(src_index, src.device), _as_index(dst_index, src.device),
                           -1 if rows is None else int(rows), error)
    return error


def accumulate_rows(src, index, out=None, error=None):
    """out[t] = sum over j of src[index[t, j]] (bf16 rows, fp32 sums).
    Returns (out, error word)."""
    if out is None:
        out = torch.empty(index.shape[0], src.shape[1], dtype=src.dtype, device=src.device)
    if not src.is_cuda:
        return out, accumulate_rows_reference(src, index, out)
    from .. import native

    if error is None:
        error = torch.zeros(1, dtype=torch.int32, device=src.device)
    native().ops.rows_accumulate(src, out, _as_index(index, src.device), error)
    return out, error


def check_error(error):
    """Raises RuntimeError if an error word (int or tensor) has bits set (synchronises)."""
    e = int(error.item()) if torch.is_tensor(error) else int(error)
    if e:
        what = [n for b, n in ((SRC_RANGE, "a source index"), (DST_RANGE, "a destination index")) if e & b]
        raise RuntimeError("row copy skipped rows: " + " and ".join(what) + " past the end of its tensor")


__all__ = ["copy_rows", "accumulate_rows", "copy_rows_reference", "accumulate_rows_reference", "check_error"]
