"""Oracle for the flat dequantization ops (test infrastructure only).

Two arithmetic definitions are provided for every format:

``contract`` -- what every reference test asserts:
    out = fp16_rn( fp32_rn( (q - z) * s ) )
    with the product evaluated exactly (it always fits a float64), rounded to
    float32, then to float16.  This is tests/test_dequant_correctness.py:18-38
    (numpy evaluates ``(nibble - zps) * scales`` in float64, stores it into a
    float32 array, and ``torch.tensor(..., dtype=float16)`` rounds float32 to
    float16).  One deviation, recorded on purpose: the reference computes
    ``np.where(nibble >= 8, nibble - 16, nibble)`` on a uint32 array
    (:35, and :58 for s3) which wraps to 2**32-1 instead of -1; here the
    nibbles are int64 so the two's-complement value is right.

``magic`` -- bit-exact with the reference GPU kernels
    (src/kernels/lop3_dequant.cu:9-123, helpers src/kernels/lop3_dequant.h:10-85):
    raw = B + q is built exactly in fp16 by a LOP3 with a magic exponent,
    bias = fp16_rn( fp32_rn( fp32_rn(-B - z) * s ) ) is computed in fp32,
    out = fp16_rn( raw * s + bias ) by one fused fp16 FMA (fma.rn.f16x2).
    B = 1024 (u4), 1032 (s4), 1028 (s3).  The product-plus-sum is exact in
    float64 (at most 50 significant bits), so one numpy float64->float16
    conversion (which rounds once, to nearest even) reproduces the FMA.

Element order within a word is natural: element j of the output is nibble j
(bits 4j..4j+3) for u4/s4 and element i (bits 3i..3i+2) for s3, as the
reference kernels store it (lop3_dequant.cu:37-44, 113-122).
"""

import numpy as np

MAGIC_BIAS = {"u4": 1024.0, "s4": 1032.0, "s3": 1028.0}
ELEMS_PER_WORD = {"u4": 8, "s4": 8, "s3": 10, "fp8": 4}


def as_u32(packed) -> np.ndarray:
    """Packed words (int32 or uint32, any shape) as non-negative int64 values.

    Going through int64 keeps bit 31 (run_empirical.py:427-440 documents the
    reference bug that dropped it)."""
    return np.asarray(packed).astype(np.int64) & 0xFFFFFFFF


def unpack_u4(packed) -> np.ndarray:
    """(n,) words -> (n, 8) nibbles 0..15; nibble j = bits 4j..4j+3."""
    w = as_u32(packed).reshape(-1)
    shifts = (4 * np.arange(8, dtype=np.int64))[None, :]
    return (w[:, None] >> shifts) & 0xF


def unpack_s4(packed) -> np.ndarray:
    """(n,) words -> (n, 8) two's-complement nibbles -8..7."""
    u = unpack_u4(packed)
    return np.where(u >= 8, u - 16, u)


def unpack_s3(packed) -> np.ndarray:
    """(n,) words -> (n, 10) signed 3-bit values -4..3; element i = bits 3i..3i+2.

    Follows tests/test_dequant_correctness.py:54-59 (with int64, see module doc)
    and src/kernels/h17_mega_kernel.h:10-21.  Bits 30-31 are ignored."""
    w = as_u32(packed).reshape(-1)
    shifts = (3 * np.arange(10, dtype=np.int64))[None, :]
    v = (w[:, None] >> shifts) & 0x7
    return np.where(v >= 4, v - 8, v)


def fp16_bits(x) -> np.ndarray:
    """float16 array -> uint16 bit patterns (for bit-exact comparisons)."""
    return np.ascontiguousarray(np.asarray(x, dtype=np.float16)).view(np.uint16)


def _per_word(vals, n, name):
    """Per-word scale / zero-point vector: numel n, or numel 1 broadcast
    (the reference oracle broadcasts size-1 tensors,
    tests/test_dequant_correctness.py:26-29)."""
    v = np.asarray(vals, dtype=np.float16).reshape(-1)
    if v.size == 1:
        return np.broadcast_to(v, (n,))
    if v.size != n:
        raise ValueError(f"{name} must have 1 or {n} elements, got {v.size}")
    return v


def _contract(q, s16, z16):
    with np.errstate(over="ignore", invalid="ignore"):
        return _contract_(q, s16, z16)


def _contract_(q, s16, z16):
    exact = (q.astype(np.float64) - z16.astype(np.float64)[:, None]) * s16.astype(np.float64)[:, None]
    return exact.astype(np.float32).astype(np.float16)


def _magic(q, s16, z16, big_b):
    with np.errstate(over="ignore", invalid="ignore"):
        return _magic_(q, s16, z16, big_b)


def _magic_(q, s16, z16, big_b):
    s32 = s16.astype(np.float32)
    z32 = z16.astype(np.float32)
    # lop3_dequant.cu:23-26 -- bias in fp32, then __float2half (round to nearest)
    bias16 = ((np.float32(-big_b) - z32) * s32).astype(np.float16)
    raw = q.astype(np.float64) + big_b                       # exact fp16 value B + q
    fused = raw * s16.astype(np.float64)[:, None] + bias16.astype(np.float64)[:, None]
    return fused.astype(np.float16)                           # one rounding == fma.rn.f16


def dequantize(kind, packed, scales, zero_points, mode="contract") -> np.ndarray:
    """Flat dequantization of u4 / s4 / s3 words with PER-WORD scale and zero
    point (lop3_dequant.cu:19-21 indexes both by word).  Returns a 1-D float16
    array of numel*8 (u4, s4) or numel*10 (s3) values, as
    bindings.cpp:18-20 / :144-146 shape the output."""
    if kind not in MAGIC_BIAS:
        raise ValueError(f"unknown kind {kind!r}")
    if mode not in ("contract", "magic"):
        raise ValueError(f"unknown mode {mode!r}")
    w = as_u32(packed).reshape(-1)
    n = w.size
    s16 = _per_word(scales, n, "scales")
    z16 = _per_word(zero_points, n, "zero_points") if np.asarray(zero_points).size else np.zeros(n, np.float16)
    if kind == "u4":
        q = unpack_u4(w)
    elif kind == "s4":
        q = unpack_s4(w)
    else:
        q = unpack_s3(w)
    if mode == "contract":
        out = _contract(q, s16, z16)
    else:
        out = _magic(q, s16, z16, MAGIC_BIAS[kind])
    return out.reshape(-1)


def _e4m3_bytes(packed):
    w = as_u32(packed).reshape(-1)
    return (w[:, None] >> (8 * np.arange(4, dtype=np.int64))[None, :]) & 0xFF


def dequantize_fp8(packed, scales, mode="contract") -> np.ndarray:
    """FP8-E4M3 bytes (4 per word, byte j = bits 8j..8j+7) -> float16.

    contract: tests/test_dequant_correctness.py:63-84 -- value is 0 when the
    exponent field is 0, else (-1)^s * 2^(e-7) * (1 + m/8); times the per-word
    scale, rounded fp32 then fp16 (the product is exact in fp32).
    magic: src/kernels/lop3_dequant.h:93-123 -- the fp16 pattern
    ((b & 0x7F) << 7) + 0x2000 | (b & 0x80) << 8, then fma.rn.f16(raw, s, +0).
    Neither handles E4M3 subnormals or NaN; both are reproduced as the
    reference has them."""
    b = _e4m3_bytes(packed)
    n = b.shape[0]
    s16 = _per_word(scales, n, "scales")
    sign = (b >> 7) & 1
    if mode == "contract":
        e = (b >> 3) & 0xF
        m = b & 0x7
        mag = np.ldexp(1.0 + m / 8.0, (e - 7).astype(np.int32))
        val = np.where(e > 0, np.where(sign == 1, -mag, mag), 0.0)
        out = (val * s16.astype(np.float64)[:, None]).astype(np.float32).astype(np.float16)
    elif mode == "magic":
        bits = (((b & 0x7F) << 7) + 0x2000) | ((b & 0x80) << 8)
        raw = bits.astype(np.uint16).view(np.float16).astype(np.float64)
        out = (raw * s16.astype(np.float64)[:, None] + 0.0).astype(np.float16)
    else:
        raise ValueError(f"unknown mode {mode!r}")
    return out.reshape(-1)
