"""Parity of the INT3 (H17 packing) prefill GEMM on tcgen05 with the oracle
(max rel err <= 1e-2 of max|y|, mean abs err <= 1e-3 of mean|y|): M > 16 at
the INT3 configuration's shapes (K = 4096 and 14336 padded to multiples of
10), groups 128 and 100 (the reference's), zero points, K % 4 != 0 (4-byte
activation copies), ragged M and N, and split K."""

import numpy as np
import pytest
import torch

import oracle
import t4_cuda_b200
import t4_kernels
from tests.test_gemv_gpu import assert_gemm_close
from tests.test_int3_gpu import make_int3

pytestmark = pytest.mark.gpu


def _dev(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def _run(dev, A, W, s, z, group):
    zt = _dev(z, dev) if z is not None else torch.empty(0, dtype=torch.float16, device=dev)
    return t4_kernels.fused_h17_gemv_s3(_dev(A, dev), _dev(W, dev), _dev(s, dev), zt, group_size=group)


@pytest.mark.parametrize("M,K,N,group,zp", [
    # single-CTA kernel (M <= 128, or an under-filled grid that splits K)
    (17, 4100, 256, 128, False),      # smallest M on the tensor cores, one tile
    (64, 4100, 512, 128, True),
    (130, 4090, 264, 100, False),     # K % 4 == 2 (4-byte copies), N tail, split K
    (256, 14340, 1024, 128, False),   # K >= 8192 with 8 tiles: split K 8 ways
    (200, 14340, 264, 100, True),     # split K, group boundaries inside steps, zero points
    (300, 1000, 512, 64, True),       # group 64: every step in one group
    (40, 650, 16, 640, True),         # one group over most of K, N = 16
    # CTA pairs (M > 128)
    (512, 4100, 4096, 128, False),    # the 4096 x 4096 projection at prefill
    (300, 4090, 4096, 100, False),    # K % 4 == 2, ragged M (the second pair holds 44 rows, all in its first CTA)
    (129, 30, 64, 100, False),        # K < one step; the pair's second CTA holds one row
    (512, 14340, 3328, 128, True),    # pairs split K in two (113 K steps each), zero points
    (2048, 4100, 2048, 128, False),
])
def test_int3_gemm_vs_oracle(cuda_device, M, K, N, group, zp):
    rng = np.random.default_rng(abs(hash(("tc", M, K, N, group, zp))) % 2 ** 32)
    A, W, s, z = make_int3(rng, M, K, N, group, zp)
    C = _run(cuda_device, A, W, s, z, group)
    assert C.shape == (M, N)
    assert_gemm_close(C, oracle.ref_int3_gemv(A, W, s, z, group), f"M={M} K={K} N={N} g={group} zp={zp}")
    assert t4_cuda_b200.device_error(cuda_device) == 0


def test_int3_gemm_full_word_range(cuda_device):
    """Words with bits 30-31 set (unused by the packing) and every 3-bit code:
    the top two bits must not leak into field 9."""
    rng = np.random.default_rng(7)
    M, K, N, group = 96, 1280, 256, 128
    A = rng.standard_normal((M, K)).astype(np.float16)
    W = rng.integers(0, 2 ** 32, size=(K // 10, N), dtype=np.int64).astype(np.uint32).view(np.int32)
    s = (np.abs(rng.standard_normal((K // group, N)) * 0.02) + 1e-3).astype(np.float16)
    C = _run(cuda_device, A, W, s, None, group)
    assert_gemm_close(C, oracle.ref_int3_gemv(A, W, s, None, group), "full word range")


def test_int3_gemm_kernel_choice(cuda_device):
    """"gemv" keeps M > 16 on the register-streaming kernel; both paths agree
    with the oracle on the same inputs."""
    rng = np.random.default_rng(11)
    M, K, N, group = 48, 4100, 512, 128
    A, W, s, z = make_int3(rng, M, K, N, group, True)
    ref = oracle.ref_int3_gemv(A, W, s, z, group)
    prev = t4_cuda_b200.set_int3_kernel("gemv")
    try:
        assert_gemm_close(_run(cuda_device, A, W, s, z, group), ref, "gemv at M = 48")
    finally:
        t4_cuda_b200.set_int3_kernel(prev)
    assert_gemm_close(_run(cuda_device, A, W, s, z, group), ref, "tcgen05 at M = 48")
    assert t4_cuda_b200.device_error(cuda_device) == 0


def test_int3_gemm_in_graph(cuda_device):
    """Split-K INT3 GEMM captured into a CUDA graph and replayed: the workspace
    counters return to zero after each launch, so replays agree."""
    rng = np.random.default_rng(5)
    M, K, N, group = 256, 14340, 512, 128
    A, W, s, z = make_int3(rng, M, K, N, group, False)
    At, Wt, st = _dev(A, cuda_device), _dev(W, cuda_device), _dev(s, cuda_device)
    zt = torch.empty(0, dtype=torch.float16, device=cuda_device)
    stream = torch.cuda.Stream(cuda_device)
    with torch.cuda.stream(stream):
        t4_kernels.fused_h17_gemv_s3(At, Wt, st, zt, group_size=group)     # workspace made before capture
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            C = t4_kernels.fused_h17_gemv_s3(At, Wt, st, zt, group_size=group)
        outs = []
        for _ in range(3):
            g.replay()
            outs.append(C.clone())
        stream.synchronize()
    ref = oracle.ref_int3_gemv(A, W, s, None, group)
    for o in outs:
        assert_gemm_close(o, ref, "graph replay")
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    del g
