"""Oracle for the H17 INT3 fused GEMV (test infrastructure only).

Layout (src/kernels/h17_mega_kernel.h:10-21, tests/test_h17_fused_int3_gemv.py:426-434):
``W_packed`` is int32 [K/10, N]; element i of word (kw, n) is K row 10*kw + i
at bits 3i..3i+2 (i = 0..9), two's complement -4..3; bits 30-31 are unused.
Scales / zero points are [G, N] with G = ceil(K / group_size); the
reference fixes group_size = 100 (h17_mega_kernel.cu:22), this library makes
it an argument (e.g. 128, where a word can straddle two groups).
"""

import numpy as np

from .dequant import as_u32


def pack_int3(q_uint) -> np.ndarray:
    """(N, K) values 0..7 -> (K/10, N) uint32 words; restates
    tests/test_h17_fused_int3_gemv.py:426-434."""
    q = np.asarray(q_uint).astype(np.uint32)
    N, K = q.shape
    if K % 10:
        raise ValueError("K must be a multiple of 10 for 10-per-uint32 packing")
    q = q.reshape(N, K // 10, 10)
    shifts = (np.arange(10, dtype=np.uint32) * 3).reshape(1, 1, 10)
    words = (q << shifts).sum(axis=2, dtype=np.uint64).astype(np.uint32)
    return np.ascontiguousarray(words.T)


def quantize_int3(W, group_size=100):
    """Affine INT3 quantizer of tests/test_h17_fused_int3_gemv.py:437-456:
    W (N, K) float32 -> packed (K/10, N) uint32, scales (G, N) f32, zp (G, N) f32
    with tc = clip(round(W/scale + zp), -4, 3) and zp = -4 - wmin/scale."""
    W = np.asarray(W, dtype=np.float32)
    N, K = W.shape
    if K % 10:
        raise ValueError("K must be a multiple of 10")
    G = (K + group_size - 1) // group_size
    pad = G * group_size - K
    if pad:
        W = np.concatenate([W, np.zeros((N, pad), dtype=np.float32)], axis=1)
    Wg = W.reshape(N, G, group_size)
    wmin = Wg.min(axis=2)
    wmax = Wg.max(axis=2)
    span = wmax - wmin
    scale = np.where(span > 0, span / 7.0, 1.0)
    zp = -4.0 - wmin / scale
    tc = np.clip(np.round(Wg / scale[:, :, None] + zp[:, :, None]), -4, 3).astype(np.int32)
    q = (tc & 0x7).astype(np.uint32).reshape(N, G * group_size)[:, :K]
    return pack_int3(q), np.ascontiguousarray(scale.T), np.ascontiguousarray(zp.T)


def unpack_int3_matrix(W_packed) -> np.ndarray:
    """int32 [K/10, N] -> int64 [K, N] two's-complement values -4..3."""
    w = as_u32(W_packed)
    KW, N = w.shape
    v = (w[:, None, :] >> (3 * np.arange(10, dtype=np.int64))[None, :, None]) & 0x7
    v = np.where(v >= 4, v - 8, v)
    return v.reshape(KW * 10, N)


def dequant_int3_matrix(W_packed, scales, zero_points=None, group_size=100) -> np.ndarray:
    """float16 [K, N] weights with w = fp16((tc - zp_g) * s_g), the product
    rounded once from double as in tests/test_h17_fused_int3_gemv.py:466-469
    (identical to the dequant contract whenever zp = 0)."""
    tc = unpack_int3_matrix(W_packed)
    K, N = tc.shape
    G = (K + group_size - 1) // group_size
    s = np.asarray(scales, dtype=np.float64).reshape(G, N)
    if zero_points is None or np.asarray(zero_points).size == 0:
        z = np.zeros((G, N))
    else:
        z = np.asarray(zero_points, dtype=np.float64).reshape(G, N)
    g = np.arange(K) // group_size
    return ((tc - z[g]) * s[g]).astype(np.float16)


def ref_int3_gemv(A, W_packed, scales, zero_points=None, group_size=100) -> np.ndarray:
    """fp32 C[M, N] = fp16(A) @ dequant(W) with fp32 accumulation -- a
    vectorised restatement of ``cpu_ref_h17_gemv``
    (tests/test_h17_fused_int3_gemv.py:459-472), whose literal triple loop is
    O(M*N*K) Python.  A may be 1-D (then M = 1, as bindings.cpp:211-213)."""
    A16 = np.asarray(A, dtype=np.float16)
    if A16.ndim == 1:
        A16 = A16[None, :]
    W16 = dequant_int3_matrix(W_packed, scales, zero_points, group_size)
    return A16.astype(np.float32) @ W16.astype(np.float32)
