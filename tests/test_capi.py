"""The C-ABI library loads, exports every entry point include/t4b200.h
declares, and rejects bad arguments with status codes before touching a GPU.
CPU only: no call here reaches a CUDA runtime function."""

import ctypes
import os
import re

import pytest

from tests.conftest import ROOT

HEADER = os.path.join(ROOT, "include", "t4b200.h")


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(t4b_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from t4_cuda_b200 import _lib
    return _lib.load()


def test_header_declares_the_seven_ops():
    names = _declared()
    for op in ("dequantize_u4", "dequantize_s4", "dequantize_s3", "dequantize_fp8",
               "fused_w4a16_gemm_u4", "fused_w4a16_gemm_s4", "fused_h17_gemv_s3"):
        assert "t4b_" + op in names


def test_library_exports_every_declared_symbol(lib):
    for name in _declared():
        assert hasattr(lib, name), name


def test_status_strings_and_version(lib):
    assert lib.t4b_status_string(0) == b"ok"
    for code in range(1, 7):
        assert lib.t4b_status_string(code) and lib.t4b_status_string(code) != b"unknown status"
    assert lib.t4b_version() >> 16 == 1
    assert lib.t4b_last_cuda_error() == 0


def _fake(addr=0x10000):
    """A non-null, 256-byte aligned address; validation fails before any use."""
    return ctypes.c_void_p(addr)


def test_dequant_argument_validation(lib):
    p = _fake()
    assert lib.t4b_dequantize_u4(p, p, p, p, -1, 1, 1, 0, None) == 1          # negative count
    assert lib.t4b_dequantize_u4(p, p, p, p, 4, 1, 1, 7, None) == 1           # bad mode
    assert lib.t4b_dequantize_s4(p, p, p, p, 0, 1, 0, 0, None) == 0           # empty is a no-op
    assert lib.t4b_dequantize_s4(None, p, p, p, 4, 4, 4, 0, None) == 2        # null words
    assert lib.t4b_dequantize_s3(p, p, None, p, 4, 4, 4, 0, None) == 2       # zero points promised, null
    assert lib.t4b_dequantize_s3(p, p, p, p, 4, 3, 4, 0, None) == 1          # scale count not 1 or n
    assert lib.t4b_dequantize_s3(p, p, p, p, 4, 4, 2, 0, None) == 1          # zero-point count
    assert lib.t4b_dequantize_u4(_fake(0x10002), p, p, p, 4, 4, 4, 0, None) == 3   # words not 4-byte aligned
    assert lib.t4b_dequantize_fp8(p, p, p, 4, 2, 0, None) == 1
    assert lib.t4b_dequantize_fp8(p, None, p, 4, 4, 0, None) == 2


def test_gemm_argument_validation(lib):
    p = _fake()
    f = lib.t4b_fused_w4a16_gemm_s4
    assert f(p, p, p, None, p, 0, 64, 64, 64, None) == 1          # M = 0
    assert f(p, p, p, None, p, 1, 64, 60, 60, None) == 1          # K % 8
    assert f(p, p, p, None, p, 1, 64, 64, 12, None) == 1          # group % 8
    assert f(p, p, p, None, p, 1, 64, 64, 48, None) == 1          # group does not divide K
    assert f(None, p, p, None, p, 1, 64, 64, 64, None) == 2
    assert f(_fake(0x10008), p, p, None, p, 1, 64, 64, 64, None) == 3   # A must be 16-byte aligned
    g = lib.t4b_fused_h17_gemv_s3
    assert g(p, p, p, None, p, 1, 64, 25, 100, None) == 1         # K % 10
    assert g(p, p, p, None, p, 1, 64, 200, 0, None) == 1          # group 0
    assert g(p, p, p, None, p, 1, 64, 200, 7, None) == 4          # group < 10 unsupported
    assert g(p, None, p, None, p, 1, 64, 200, 100, None) == 2


def test_noalloc_gemv_argument_validation(lib):
    p = _fake()
    f = lib.t4b_fused_w4a16_gemv_noalloc
    assert f(p, p, p, None, p, 0, 64, 64, 64, 1, None) == 1       # M = 0
    assert f(p, p, p, None, p, 1, 64, 60, 60, 1, None) == 1       # K % 8
    assert f(None, p, p, None, p, 1, 64, 64, 64, 1, None) == 2
    assert f(_fake(0x10008), p, p, None, p, 1, 64, 64, 64, 0, None) == 3   # A must be 16-byte aligned
    assert f(p, p, p, None, p, 17, 64, 64, 64, 1, None) == 4      # M > 16 is not a decode shape
    assert f(p, p, p, None, p, 1, 62, 64, 64, 1, None) == 4       # N % 4


def test_grouped_gemm_argument_validation(lib):
    p = _fake()
    vp2 = ctypes.c_void_p * 2
    ptrs = vp2(0x10000, 0x20000)
    Ns = (ctypes.c_int * 2)(64, 64)
    f = lib.t4b_fused_w4a16_gemm_grouped
    assert f(p, 0, ptrs, ptrs, None, ptrs, Ns, 1, 64, 64, 1, None) == 1        # no projection
    assert f(p, 5, ptrs, ptrs, None, ptrs, Ns, 1, 64, 64, 1, None) == 1        # more than T4B_GROUPED_MAX
    assert f(p, 2, ptrs, ptrs, None, ptrs, Ns, 0, 64, 64, 1, None) == 1        # M = 0
    assert f(p, 2, ptrs, ptrs, None, ptrs, Ns, 1, 64, 48, 1, None) == 1        # group does not divide K
    assert f(p, 2, ptrs, ptrs, None, ptrs, (ctypes.c_int * 2)(64, 0), 1, 64, 64, 1, None) == 1   # N = 0
    assert f(None, 2, ptrs, ptrs, None, ptrs, Ns, 1, 64, 64, 1, None) == 2     # null A
    assert f(p, 2, None, ptrs, None, ptrs, Ns, 1, 64, 64, 1, None) == 2        # null weight list
    assert f(p, 2, vp2(0x10000, None), ptrs, None, ptrs, Ns, 1, 64, 64, 1, None) == 2   # null weight
    assert f(p, 2, ptrs, ptrs, vp2(0x10000, None), ptrs, Ns, 1, 64, 64, 1, None) == 2   # zero points: all or none
    assert f(_fake(0x10008), 2, ptrs, ptrs, None, ptrs, Ns, 1, 64, 64, 1, None) == 3   # A 16-byte aligned
    assert f(p, 2, vp2(0x10000, 0x20002), ptrs, None, ptrs, Ns, 1, 64, 64, 1, None) == 3   # W 4-byte aligned
    plan = lib.t4b_fused_w4a16_gemm_grouped_plan
    ctas = (ctypes.c_int * 2)()
    assert plan(0, Ns, 1, 64, 64, 0, ctas) == 1
    assert plan(2, Ns, 1, 60, 60, 0, ctas) == 1                                 # K % 8
    assert plan(2, None, 1, 64, 64, 0, ctas) == 2
    assert plan(2, Ns, 17, 64, 64, 0, ctas) == 4                                # M > 16: one launch each
