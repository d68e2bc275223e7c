"""The allocation-free grouped GEMM entry point, called through its exported C
symbol, against the regular entry point (kiwi_b200._C.ops.GroupedGemm).

The C entry point exists for callers that may not allocate device memory
while running (engines that pre-reserve the whole GPU for their own pool,
hosts without PyTorch's allocator); it keeps its scratch in a fixed device
array.  This file is
named to be collected last.
"""
import ctypes
import glob
import os

import pytest
import torch

import kiwi_b200

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
    return lib, fn


def _call(fn, a, b, groups, n, k, counts, out, swiglu, scale):
    stream = torch.cuda.current_stream().cuda_stream
    return fn(a.data_ptr(), a.shape[0], b.data_ptr(), groups, n, k, counts.data_ptr(), out.data_ptr(),
              out.shape[0], 1 if swiglu else 0, scale.data_ptr() if scale is not None else None, stream)


@pytest.mark.parametrize("swiglu", [False, True])
def test_noalloc_matches_regular_entry_point_twice(swiglu):
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
        torch.cuda.synchronize()
        tol = 2e-2 * ref.float().abs().max().item() + 1e-2
        assert (got.float() - ref.float()).abs().max().item() <= tol, f"call {call}"


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
