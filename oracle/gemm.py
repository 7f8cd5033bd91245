"""Oracle for the fused W4A16 GEMV / GEMM (test infrastructure only).

Layout (src/kernels/fused_w4a16_gemm.cu:48-61 and the reference CPU check
tests/test_fused_gemm_correctness.py:11-31): ``W_packed`` is int32 [K/8, N]
row-major; word (kw, n) holds K rows 8*kw + j in nibble j (bits 4j..4j+3).

The reference GEMM oracle is ``matmul(A.float(), dequant(W).half().float())``
(tests/test_fused_gemm_correctness.py:33-36): weights rounded to fp16 by the
contract rule, products and sums in fp32.  ``ref_w4_gemm`` restates it.

Scales / zero points: the reference kernel takes one value per output column,
shape (1, N) or (N,) (fused_w4a16_gemm.cu:31-32).  This library also accepts a
grouped shape (K/g, N): group g of column n covers K rows [g*gs, (g+1)*gs).
A per-column tensor is the special case of one group of size K.
"""

import numpy as np

from .dequant import as_u32


def pack_int4(q, signed=True) -> np.ndarray:
    """Pack integer weights q[K, N] (values -8..7 if signed, else 0..15) into
    int32 words [K/8, N] with K row 8*kw + j in nibble j -- the inverse of
    tests/test_fused_gemm_correctness.py:11-20."""
    q = np.asarray(q, dtype=np.int64)
    K, N = q.shape
    if K % 8:
        raise ValueError("K must be a multiple of 8")
    nib = (q & 0xF).reshape(K // 8, 8, N)
    words = np.zeros((K // 8, N), dtype=np.int64)
    for j in range(8):
        words |= nib[:, j, :] << (4 * j)
    return words.astype(np.uint32).view(np.int32)


def unpack_w4_matrix(W_packed, signed) -> np.ndarray:
    """int32 [K/8, N] -> int64 [K, N] (row 8*kw + j = nibble j of word kw)."""
    w = as_u32(W_packed)
    KW, N = w.shape
    nib = (w[:, None, :] >> (4 * np.arange(8, dtype=np.int64))[None, :, None]) & 0xF
    if signed:
        nib = np.where(nib >= 8, nib - 16, nib)
    return nib.reshape(KW * 8, N)


def expand_scales(vals, K, N, name="scales"):
    """Scale / zero-point tensor of shape (N,), (1, N) or (G, N) -> (G, N)
    float16 plus the group size K // G.  ``None`` or an empty tensor (zero
    points only) -> zeros with G = 1."""
    if vals is None or np.asarray(vals).size == 0:
        return np.zeros((1, N), np.float16), K
    v = np.asarray(vals, dtype=np.float16)
    if v.ndim == 1:
        v = v.reshape(1, -1)
    if v.ndim != 2 or v.shape[1] != N:
        raise ValueError(f"{name} must have shape (N,), (1, N) or (K/g, N); got {v.shape}")
    G = v.shape[0]
    if K % G:
        raise ValueError(f"{name}: {G} groups do not divide K={K}")
    return v, K // G


def dequant_w4_matrix(W_packed, scales, zero_points=None, signed=True) -> np.ndarray:
    """Contract dequantization of a packed weight matrix -> float16 [K, N]:
    fp16_rn(fp32_rn((q - z) * s)) per element, with the group of row k being
    k // group_size (tests/test_fused_gemm_correctness.py:22-31)."""
    q = unpack_w4_matrix(W_packed, signed)
    K, N = q.shape
    s, gs = expand_scales(scales, K, N, "scales")
    z, gz = expand_scales(zero_points, K, N, "zero_points")
    s_k = np.repeat(s.astype(np.float64), gs, axis=0)
    z_k = np.repeat(z.astype(np.float64), gz, axis=0)
    exact = (q.astype(np.float64) - z_k) * s_k
    return exact.astype(np.float32).astype(np.float16)


def ref_w4_gemm(A, W_packed, scales, zero_points=None, signed=True) -> np.ndarray:
    """fp32 C[M, N] = A.float() @ dequant(W).float() (the reference's
    ``cpu_reference_gemm`` before its final ``.half()``,
    tests/test_fused_gemm_correctness.py:33-36)."""
    A32 = np.asarray(A, dtype=np.float16).astype(np.float32)
    if A32.ndim == 1:
        A32 = A32[None, :]
    W32 = dequant_w4_matrix(W_packed, scales, zero_points, signed).astype(np.float32)
    return A32 @ W32
