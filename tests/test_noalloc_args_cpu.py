"""The allocation-free GEMM entry point (C symbol kiwi_grouped_gemm_bf16_noalloc)
rejects bad arguments with its documented codes before it touches a device,
so these run without a GPU.  No pointer passed here is ever dereferenced:
every call fails one of the argument checks first."""
import ctypes
import glob
import os

import pytest

import kiwi_b200

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    kiwi_b200.native()
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
    return lib


OK_PTR = 1 << 20  # a 16-byte-aligned address value (never dereferenced: each call fails a check first)


@pytest.mark.parametrize("groups,n,k,a,c,rows,code,words", [
    (0, 256, 64, OK_PTR, OK_PTR, 8, 1, "num_groups"),
    (1025, 256, 64, OK_PTR, OK_PTR, 8, 1, "num_groups"),
    (2, 200, 64, OK_PTR, OK_PTR, 8, 2, "multiple of 256"),
    (2, 256, 48, OK_PTR, OK_PTR, 8, 2, "multiple of 256"),
    (2, 256, 64, None, OK_PTR, 8, 3, "null pointer"),
    (2, 256, 64, OK_PTR, OK_PTR, 0, 3, "empty"),
    (2, 256, 64, OK_PTR + 8, OK_PTR, 8, 4, "16-byte aligned"),
    (2, 256, 64, OK_PTR, OK_PTR + 2, 8, 4, "16-byte aligned"),
])
def test_argument_checks(lib, groups, n, k, a, c, rows, code, words):
    fn = lib.kiwi_grouped_gemm_bf16_noalloc
    rc = fn(a, rows, OK_PTR, groups, n, k, OK_PTR, c, rows, 0, None, None)
    assert rc == code
    assert words in lib.kiwi_noalloc_last_error().decode()


def test_max_groups(lib):
    assert lib.kiwi_noalloc_max_groups() == 1024


def test_error_word_reader_rejects_a_null_destination(lib):
    """kiwi_noalloc_error_word checks its host pointer before any CUDA call."""
    fn = lib.kiwi_noalloc_error_word
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    assert fn(None, None) == 3
    assert "null host_out" in lib.kiwi_noalloc_last_error().decode()


def test_header_declares_every_exported_symbol():
    """include/kiwi/gemm/noalloc.h declares the four C symbols the library exports."""
    text = open(os.path.join(ROOT, "include", "kiwi", "gemm", "noalloc.h")).read()
    for name in ("kiwi_noalloc_max_groups", "kiwi_noalloc_last_error", "kiwi_grouped_gemm_bf16_noalloc",
                 "kiwi_noalloc_error_word"):
        assert name + "(" in text
