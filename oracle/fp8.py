"""Oracle for the FP8-E4M3 weight GEMM (test infrastructure only).

The reference has no fused FP8 op; its FP8 format is the flat dequantizer's
(src/kernels/lop3_dequant.h:93-123, bindings.cpp:161-183): four E4M3 bytes per
int32 word, byte j at bits 8j..8j+7.  The fused op packs K row 4 kw + j of
column n into byte j of word (kw, n) -- the INT4 GEMM's layout
(tests/test_fused_gemm_correctness.py:11-15) with bytes for nibbles.

E4M3 is decoded exactly (the OCP 8-bit floating-point format, as
torch.float8_e4m3fn): sign bit 7, exponent bits 3-6 (bias 7), mantissa bits
0-2; exponent 0 is subnormal (m / 8 * 2^-6); 0x7F / 0xFF are NaN; there is no
infinity.  The reference's CPU dequant (tests/test_dequant_correctness.py:63-84)
differs on those 16 codes (it flushes subnormals to 0 and reads the NaN codes
as +-480); the fused op follows the format, not that deviation.

The weight is fp16_rn(fp32(e4m3 * s)) -- the product is exact in fp32 -- and
the GEMM is fp32 A @ W, as ref_w4_gemm does for INT4.
"""

import numpy as np

from .gemm import expand_scales


def e4m3_to_float(codes) -> np.ndarray:
    """uint8 codes -> float64 values (NaN for 0x7F / 0xFF)."""
    b = np.asarray(codes, dtype=np.int64) & 0xFF
    sign = np.where(b >> 7, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = (b & 0x7).astype(np.float64)
    mag = np.where(e == 0, np.ldexp(m / 8.0, -6), np.ldexp(1.0 + m / 8.0, (e - 7).astype(np.int32)))
    out = sign * mag
    return np.where((b & 0x7F) == 0x7F, np.nan, out)


def pack_fp8(codes) -> np.ndarray:
    """uint8 codes [K, N] -> int32 words [K/4, N] (byte j of word kw = row 4 kw + j)."""
    c = np.asarray(codes, dtype=np.int64) & 0xFF
    K, N = c.shape
    if K % 4:
        raise ValueError("K must be a multiple of 4")
    c = c.reshape(K // 4, 4, N)
    words = c[:, 0] | (c[:, 1] << 8) | (c[:, 2] << 16) | (c[:, 3] << 24)
    return words.astype(np.uint32).view(np.int32)


def unpack_fp8_codes(W_packed) -> np.ndarray:
    """int32 words [K/4, N] -> uint8 codes [K, N]."""
    w = np.asarray(W_packed).view(np.uint32).astype(np.int64)
    KW, N = w.shape
    b = (w[:, None, :] >> (8 * np.arange(4, dtype=np.int64))[None, :, None]) & 0xFF
    return b.reshape(KW * 4, N)


def dequant_fp8_matrix(W_packed, scales) -> np.ndarray:
    """fp16 [K, N] weights fp16_rn(fp32(e4m3 * s)), group of row k = k // group."""
    v = e4m3_to_float(unpack_fp8_codes(W_packed))
    K, N = v.shape
    s, gs = expand_scales(scales, K, N, "scales")
    s_k = np.repeat(s.astype(np.float64), gs, axis=0)
    with np.errstate(invalid="ignore"):
        return (v * s_k).astype(np.float32).astype(np.float16)


def ref_fp8_gemm(A, W_packed, scales) -> np.ndarray:
    """fp32 C[M, N] = A.float() @ dequant_fp8(W).float()."""
    A32 = np.asarray(A, dtype=np.float16).astype(np.float32)
    if A32.ndim == 1:
        A32 = A32[None, :]
    W32 = dequant_fp8_matrix(W_packed, scales).astype(np.float32)
    with np.errstate(invalid="ignore"):
        return A32 @ W32
