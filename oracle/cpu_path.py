"""The reference's CPU dequant + matmul path, restated with torch on the host
cores (test / baseline infrastructure only).

tests/test_fused_gemm_correctness.py:11-36 is the reference's CPU
implementation of this path: unpack the nibbles with shifts and masks,
``(q - z) * s`` in fp32, ``.half()``, then ``torch.matmul(A.float(), W.float())``.
``w4_gemm`` does the same operations on whole tensors (the reference loops
over the 8 nibble positions, as does this); ``int3_gemv`` is the numpy-style
restatement of tests/test_h17_fused_int3_gemv.py:459-472 in torch, since the
literal triple loop is O(M*N*K) Python.

bench.py times these as the CPU baseline ("kind": "port") and as the
``--impl reference`` arm.
"""

import torch


def unpack_w4(W_packed, signed):
    """int32 [K/8, N] -> int8/uint8 [K, N]; row 8*kw + j = nibble j
    (tests/test_fused_gemm_correctness.py:11-20)."""
    KW, N = W_packed.shape
    out = torch.empty((KW * 8, N), dtype=torch.int16)
    for i in range(8):
        out[i::8, :] = (W_packed >> (4 * i)) & 0xF
    if signed:
        out = torch.where(out >= 8, out - 16, out)
    return out


def dequant_w4(W_packed, scales, zero_points, signed):
    """fp16 [K, N] = ((q - z) * s).half() with per-group scale rows
    (tests/test_fused_gemm_correctness.py:22-31, generalised to (K/g, N))."""
    q = unpack_w4(W_packed, signed).float()
    K, N = q.shape
    s = scales.float().reshape(-1, N)
    g = K // s.shape[0]
    if g != K:
        s = s.repeat_interleave(g, dim=0)
    if zero_points is not None and zero_points.numel():
        z = zero_points.float().reshape(-1, N)
        if z.shape[0] != K:
            z = z.repeat_interleave(K // z.shape[0], dim=0)
        q = q - z
    return (q * s).half()


def w4_gemm(A, W_packed, scales, zero_points=None, signed=True):
    """fp32 C = A.float() @ dequant(W).float() on the CPU."""
    return torch.matmul(A.float(), dequant_w4(W_packed, scales, zero_points, signed).float())


def int3_gemv(A, W_packed, scales, zero_points=None, group_size=100):
    KW, N = W_packed.shape
    K = KW * 10
    v = torch.empty((K, N), dtype=torch.int16)
    for i in range(10):
        v[i::10, :] = (W_packed >> (3 * i)) & 0x7
    tc = torch.where(v >= 4, v - 8, v).double()
    g = torch.arange(K) // group_size
    s = scales.double().reshape(-1, N)[g]
    z = zero_points.double().reshape(-1, N)[g] if zero_points is not None and zero_points.numel() else 0.0
    Wd = ((tc - z) * s).half()
    A2 = A.reshape(-1, K).half().float()
    return A2 @ Wd.float()
