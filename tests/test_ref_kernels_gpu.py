"""Parity against the reference's OWN CUDA kernels, run on this GPU.

oracle/build_ref.sh compiles the reference's unmodified kernel sources
(src/kernels/lop3_dequant.cu, fused_w4a16_gemm.cu, h17_mega_kernel.cu) for
sm_100a into oracle/_ref/libt4ref.so; the library travels with the working
tree.  These tests pin two things on real hardware:

* "magic" mode of the dequant ops (and the oracle's float64 emulation of it)
  is bit-identical to the reference GPU kernels for arbitrary fp16 scales and
  zero points (lop3_dequant.cu:9-146);
* the fused W4A16 GEMV and the H17 INT3 GEMV agree with the reference kernels
  (fused_w4a16_gemm.cu:15-222, h17_mega_kernel.cu:24-141).  The reference
  rounds each weight with its fp16 FMA and each product to fp16; with
  power-of-two scales and integer zero points both roundings of the weight are
  exact, so the contract weights equal the reference's and the only difference
  left is its fp16 product rounding and summation order: gate max |dy| <=
  2e-3 max |y|.

Inputs honour the reference kernels' unchecked contracts (full per-word
scale arrays, N % 4 == 0, K % 10 == 0 with ceil(K/100) scale rows).
"""

import ctypes
import os

import numpy as np
import pytest
import torch

import oracle
import t4_kernels

pytestmark = pytest.mark.gpu

LIB_PATH = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref", "libt4ref.so")
GATE = 2e-3


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(LIB_PATH):
        pytest.skip("oracle/_ref/libt4ref.so not built (oracle/build_ref.sh needs the reference checkout)")
    lib = ctypes.CDLL(LIB_PATH)
    vp, i32 = ctypes.c_void_p, ctypes.c_int
    lib.t4ref_dequant.argtypes = [i32, vp, vp, vp, vp, i32, vp]
    lib.t4ref_fused_w4a16.argtypes = [i32, vp, vp, vp, vp, vp, i32, i32, i32, vp]
    lib.t4ref_h17_gemv.argtypes = [vp, vp, vp, vp, vp, i32, i32, i32, i32, vp]
    for f in (lib.t4ref_dequant, lib.t4ref_fused_w4a16, lib.t4ref_h17_gemv):
        f.restype = i32
    return lib


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _t(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def _words(rng, n):
    return rng.integers(0, 2 ** 32, size=n, dtype=np.int64).astype(np.uint32).view(np.int32)


@pytest.mark.parametrize("kind,per_word,code", [("u4", 8, 0), ("s4", 8, 1), ("s3", 10, 2)])
def test_magic_dequant_bit_exact_vs_reference_kernel(cuda_device, ref, kind, per_word, code):
    rng = np.random.default_rng(100 + code)
    n = 40000 + 7
    w = _words(rng, n)
    if kind == "s3":
        w = (w.view(np.uint32) & np.uint32(0x3FFFFFFF)).view(np.int32)
    s = (rng.standard_normal(n) * 0.1).astype(np.float16)
    z = (rng.standard_normal(n) * 4).astype(np.float16)
    wt, st, zt = _t(w, cuda_device), _t(s, cuda_device), _t(z, cuda_device)
    out_ref = torch.empty(n * per_word, dtype=torch.float16, device=cuda_device)
    assert ref.t4ref_dequant(code, _p(wt), _p(out_ref), _p(st), _p(zt), n, _stream(cuda_device)) == 0
    ours = getattr(t4_kernels, f"dequantize_{kind}")(wt, st, zt, mode="magic")
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(ours.view(torch.int16), out_ref.view(torch.int16))
    emu = oracle.dequantize(kind, w, s, z, mode="magic")
    assert np.array_equal(emu.view(np.int16), out_ref.cpu().numpy().view(np.int16))


def test_fp8_dequant_bit_exact_vs_reference_kernel(cuda_device, ref):
    rng = np.random.default_rng(104)
    n = 30011
    w = _words(rng, n)
    s = (rng.standard_normal(n) * 0.5).astype(np.float16)
    wt, st = _t(w, cuda_device), _t(s, cuda_device)
    out_ref = torch.empty(n * 4, dtype=torch.float16, device=cuda_device)
    assert ref.t4ref_dequant(3, _p(wt), _p(out_ref), _p(st), ctypes.c_void_p(0), n, _stream(cuda_device)) == 0
    ours = t4_kernels.dequantize_fp8(wt, st, mode="magic")
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(ours.view(torch.int16), out_ref.view(torch.int16))


def _pow2_scales(rng, shape):
    e = rng.integers(-9, -3, size=shape)
    sign = np.where(rng.random(shape) < 0.2, -1.0, 1.0)
    return (sign * np.exp2(e)).astype(np.float16)


def _close(ours, theirs, what):
    a = ours.float().cpu().numpy()
    b = theirs.float().cpu().numpy()
    assert np.all(np.isfinite(a)) and np.all(np.isfinite(b)), what
    d = np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)
    assert d <= GATE, f"{what}: max |dy| / max |y_ref| = {d:.3e}"


@pytest.mark.parametrize("signed", [True, False])
@pytest.mark.parametrize("M,K,N,zp", [(1, 4096, 4096, False), (4, 4096, 1024, True), (8, 1024, 4096, False),
                                      (16, 2048, 512, True), (64, 1024, 1024, True), (256, 512, 768, False)])
def test_fused_w4a16_vs_reference_kernel(cuda_device, ref, signed, M, K, N, zp):
    """Per-column scales and zero points, the reference kernel's own format
    (fused_w4a16_gemm.cu:31-32); M > 16 takes the tcgen05 GEMM here."""
    rng = np.random.default_rng(M * 131 + N + (7 if signed else 0))
    A = rng.standard_normal((M, K)).astype(np.float16)
    W = rng.integers(0, 2 ** 32, size=(K // 8, N), dtype=np.int64).astype(np.uint32).view(np.int32)
    s = _pow2_scales(rng, (1, N))
    z = rng.integers(-3, 12, size=(1, N)).astype(np.float16) if zp else np.zeros((1, N), np.float16)
    At, Wt, st, zt = (_t(x, cuda_device) for x in (A, W, s, z))
    C_ref = torch.empty((M, N), dtype=torch.float16, device=cuda_device)
    assert ref.t4ref_fused_w4a16(1 if signed else 0, _p(At), _p(Wt), _p(st), _p(zt), _p(C_ref), M, N, K,
                                 _stream(cuda_device)) == 0
    op = t4_kernels.fused_w4a16_gemm_s4 if signed else t4_kernels.fused_w4a16_gemm_u4
    C = op(At, Wt, st, zt if zp else None)
    torch.cuda.synchronize(cuda_device)
    _close(C, C_ref, f"w4a16 signed={signed} M={M} K={K} N={N} zp={zp}")


@pytest.mark.parametrize("M,K,N,zp", [(1, 4100, 1024, False), (1, 1000, 4096, True), (4, 2000, 512, True)])
def test_h17_vs_reference_kernel(cuda_device, ref, M, K, N, zp):
    """Group 100 (h17_mega_kernel.cu:22), 10 INT3 per word."""
    rng = np.random.default_rng(K + N + M)
    G = -(-K // 100)
    A = rng.standard_normal((M, K)).astype(np.float16)
    W = (rng.integers(0, 2 ** 30, size=(K // 10, N), dtype=np.int64)).astype(np.uint32).view(np.int32)
    s = _pow2_scales(rng, (G, N))
    z = rng.integers(-2, 3, size=(G, N)).astype(np.float16) if zp else None
    At, Wt, st = _t(A, cuda_device), _t(W, cuda_device), _t(s, cuda_device)
    zt = _t(z, cuda_device) if zp else None
    C_ref = torch.empty((M, N), dtype=torch.float16, device=cuda_device)
    assert ref.t4ref_h17_gemv(_p(At), _p(Wt), _p(st), _p(zt), _p(C_ref), M, N, K, G, _stream(cuda_device)) == 0
    C = t4_kernels.fused_h17_gemv_s3(At, Wt, st, zt if zp else torch.empty(0, dtype=torch.float16, device=cuda_device),
                                     group_size=100)
    torch.cuda.synchronize(cuda_device)
    _close(C, C_ref, f"h17 M={M} K={K} N={N} zp={zp}")
