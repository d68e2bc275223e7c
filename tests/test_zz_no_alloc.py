"""The allocation-free grouped GEMM entry point, called through its exported C
symbols (declared in include/kiwi/gemm/noalloc.h), against the regular entry
point (kiwi_b200._C.ops.GroupedGemm) and the fp32 reference.

The C entry point is for callers that may not allocate device memory once they
run: a serving engine that reserved the whole GPU for its own pool at start-up,
or a C host without PyTorch's caching allocator.  It keeps its scratch in one
fixed device array that every call shares.  This file is named to be collected
last, so a run that stops at its first failure has run every other test.
"""
import ctypes
import glob
import os

import pytest
import torch

import kiwi_b200
from kiwi_b200.ops import grouped_gemm_reference

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _lib():
    kiwi_b200.native()  # loads the extension (and torch's libraries) first
    so = sorted(glob.glob(os.path.join(ROOT, "kiwi_b200", "_C*.so")))
    assert so, "extension not built"
    lib = ctypes.CDLL(so[0])
    fn = lib.kiwi_grouped_gemm_bf16_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
                   ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32,
                   ctypes.c_void_p, ctypes.c_void_p]
    lib.kiwi_noalloc_last_error.restype = ctypes.c_char_p
    lib.kiwi_noalloc_max_groups.restype = ctypes.c_int
    lib.kiwi_noalloc_error_word.restype = ctypes.c_int
    lib.kiwi_noalloc_error_word.argtypes = [ctypes.POINTER(ctypes.c_int32), ctypes.c_void_p]
    return lib, fn


def _call(fn, a, b, groups, n, k, counts, out, swiglu, scale, c_rows=None):
    stream = torch.cuda.current_stream().cuda_stream
    return fn(a.data_ptr(), a.shape[0], b.data_ptr(), groups, n, k, counts.data_ptr(), out.data_ptr(),
              out.shape[0] if c_rows is None else c_rows, 1 if swiglu else 0,
              scale.data_ptr() if scale is not None else None, stream)


def _error_word(lib):
    word = ctypes.c_int32(-1)
    rc = lib.kiwi_noalloc_error_word(ctypes.byref(word), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.kiwi_noalloc_last_error()
    return word.value


@pytest.mark.parametrize("swiglu", [False, True])
def test_noalloc_matches_regular_entry_point_twice(swiglu):
    """Two calls in a row with different group sizes: each result equals the
    regular entry point's and the fp32 reference within the GEMM tests'
    tolerance, and the error word reads 0 after each."""
    lib, fn = _lib()
    C = kiwi_b200.native()
    torch.manual_seed(1)
    k, n = 512, 512
    for call, counts_list in enumerate([[70, 0, 200, 5], [1, 129, 64, 300]]):
        groups = len(counts_list)
        rows = sum(counts_list)
        a = (torch.randn(rows, k, device="cuda") * 0.5).bfloat16()
        b = (torch.randn(groups * n, k, device="cuda") * 0.05).bfloat16()
        counts = torch.tensor(counts_list, dtype=torch.int32, device="cuda")
        scale = torch.rand(rows, device="cuda") + 0.5
        cols = n // 2 if swiglu else n
        ref = torch.zeros(rows, cols, device="cuda", dtype=torch.bfloat16)
        C.ops.GroupedGemm(a, b, groups).run(counts, ref, swiglu, scale)
        got = torch.zeros(rows, cols, device="cuda", dtype=torch.bfloat16)
        rc = _call(fn, a, b, groups, n, k, counts, got, swiglu, scale)
        assert rc == 0, lib.kiwi_noalloc_last_error()
        assert _error_word(lib) == 0
        exact = grouped_gemm_reference(a, b, counts_list, swiglu=swiglu, row_scale=scale)
        tol = 2e-2 * exact.abs().max().item() + 1e-2
        assert (got.float() - ref.float()).abs().max().item() <= tol, f"call {call} vs the regular entry"
        assert (got.float() - exact).abs().max().item() <= tol, f"call {call} vs the fp32 reference"


def test_noalloc_allocates_no_device_memory():
    """After a first call (which resolves the array's address), further calls
    change neither the device's free memory nor torch's allocated bytes."""
    lib, fn = _lib()
    torch.manual_seed(2)
    k, n, counts_list = 256, 256, [40, 300, 0, 88]
    rows = sum(counts_list)
    a = torch.randn(rows, k, device="cuda").bfloat16()
    b = (torch.randn(len(counts_list) * n, k, device="cuda") * 0.05).bfloat16()
    counts = torch.tensor(counts_list, dtype=torch.int32, device="cuda")
    out = torch.zeros(rows, n, device="cuda", dtype=torch.bfloat16)
    assert _call(fn, a, b, len(counts_list), n, k, counts, out, False, None) == 0, lib.kiwi_noalloc_last_error()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    alloc0 = torch.cuda.memory_allocated()
    for _ in range(5):
        assert _call(fn, a, b, len(counts_list), n, k, counts, out, False, None) == 0
        assert _error_word(lib) == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert torch.cuda.memory_allocated() == alloc0


def test_noalloc_leaves_rows_past_c_rows_untouched():
    """With c_rows below the rows the counts describe, rows [0, c_rows) match the
    reference and the rest of the buffer keeps its contents; row_scale is read
    for rows below c_rows only (it is given exactly c_rows entries)."""
    lib, fn = _lib()
    torch.manual_seed(3)
    k, n, counts_list = 256, 256, [100, 150, 60]
    rows = sum(counts_list)
    c_rows = 180
    a = torch.randn(rows, k, device="cuda").bfloat16()
    b = (torch.randn(len(counts_list) * n, k, device="cuda") * 0.05).bfloat16()
    counts = torch.tensor(counts_list, dtype=torch.int32, device="cuda")
    scale = torch.rand(c_rows, device="cuda") + 0.5
    sentinel = torch.full((rows, n), 7.0, device="cuda", dtype=torch.bfloat16)
    out = sentinel.clone()
    rc = _call(fn, a, b, len(counts_list), n, k, counts, out, False, scale, c_rows=c_rows)
    assert rc == 0, lib.kiwi_noalloc_last_error()
    assert _error_word(lib) == 0
    full_scale = torch.cat([scale, torch.ones(rows - c_rows, device="cuda")])
    exact = grouped_gemm_reference(a, b, counts_list, row_scale=full_scale)[:c_rows]
    tol = 2e-2 * exact.abs().max().item() + 1e-2
    assert (out[:c_rows].float() - exact).abs().max().item() <= tol
    assert torch.equal(out[c_rows:], sentinel[c_rows:])


def test_noalloc_rejects_too_many_groups():
    lib, fn = _lib()
    maxg = lib.kiwi_noalloc_max_groups()
    assert maxg == 1024
    a = torch.zeros(128, 64, device="cuda", dtype=torch.bfloat16)
    b = torch.zeros((maxg + 1) * 256, 64, device="cuda", dtype=torch.bfloat16)
    counts = torch.zeros(maxg + 1, dtype=torch.int32, device="cuda")
    out = torch.zeros(128, 256, device="cuda", dtype=torch.bfloat16)
    rc = _call(fn, a, b, maxg + 1, 256, 64, counts, out, False, None)
    assert rc != 0
    assert b"num_groups must be in [1, 1024]" in lib.kiwi_noalloc_last_error()


def test_noalloc_and_regular_entry_on_two_devices():
    """One process drives two GPUs in turn (0, 1, 0, 1): the raised shared-memory
    limit, the SM count and the no-alloc scratch array are kept per device, so
    the 1-SM and 2-SM kernels and the no-alloc entry run on the second device
    after the first and each result matches the fp32 reference."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs in one process")
    lib, fn = _lib()
    C = kiwi_b200.native()
    k, n, counts_list = 256, 512, [100, 0, 257, 31]
    rows, groups = sum(counts_list), len(counts_list)
    for call, dev in enumerate((0, 1, 0, 1)):
        with torch.cuda.device(dev):
            torch.manual_seed(10 + call)
            a = (torch.randn(rows, k, device="cuda") * 0.5).bfloat16()
            b = (torch.randn(groups * n, k, device="cuda") * 0.05).bfloat16()
            counts = torch.tensor(counts_list, dtype=torch.int32, device="cuda")
            exact = grouped_gemm_reference(a, b, counts_list, swiglu=True)
            tol = 2e-2 * exact.abs().max().item() + 1e-2
            plan = C.ops.GroupedGemm(a, b, groups)
            for pair in (False, True):
                got = torch.zeros(rows, n // 2, device="cuda", dtype=torch.bfloat16)
                plan.run(counts, got, True, None, 0, pair)
                assert (got.float() - exact).abs().max().item() <= tol, f"device {dev}, pair={pair}"
            got = torch.zeros(rows, n // 2, device="cuda", dtype=torch.bfloat16)
            assert _call(fn, a, b, groups, n, k, counts, got, True, None) == 0, lib.kiwi_noalloc_last_error()
            assert _error_word(lib) == 0
            assert (got.float() - exact).abs().max().item() <= tol, f"device {dev}, no-alloc entry"
