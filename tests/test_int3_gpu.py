"""Parity of the H17 INT3 GEMV with the oracle (same gates as the W4A16 GEMM:
max rel err <= 1e-2 of max|y|, mean abs err <= 1e-3 of mean|y|) and with the
reference's own gate data (max abs <= 2.0, tests/test_h17_fused_int3_gemv.py:520-526)."""

import os

import numpy as np
import pytest
import torch

import oracle
import t4_cuda_b200
import t4_kernels
from tests.conftest import GOLDEN
from tests.test_gemv_gpu import assert_gemm_close

pytestmark = pytest.mark.gpu


def _dev(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


@pytest.mark.parametrize("tag", ["gate", "g128", "nozp"])
def test_reference_gate_cases(cuda_device, tag):
    d = np.load(os.path.join(GOLDEN, "int3_cases.npz"))
    g = int(d[tag + "_group"])
    A16 = d[tag + "_A"].astype(np.float16)
    s16 = d[tag + "_s"].astype(np.float16)
    z16 = d[tag + "_z"].astype(np.float16)
    zt = _dev(z16, cuda_device) if tag != "nozp" else torch.empty(0, dtype=torch.float16, device=cuda_device)
    C = t4_kernels.fused_h17_gemv_s3(_dev(A16, cuda_device), _dev(d[tag + "_W"], cuda_device),
                                     _dev(s16, cuda_device), zt, group_size=g)
    assert C.shape == A16.shape[:1] + (d[tag + "_W"].shape[1],)
    y = C.float().cpu().numpy()
    ref = d[tag + "_c"]          # the reference oracle, fed fp32 scales / zero points
    assert np.abs(y - ref).max() <= 2.0
    assert np.abs(ref).max() > 1e-3
    # strict gate against the oracle fed exactly what the kernel sees
    assert_gemm_close(C, oracle.ref_int3_gemv(A16, d[tag + "_W"], s16, z16 if tag != "nozp" else None, g), tag)


def make_int3(rng, M, K, N, group, zp):
    A = rng.standard_normal((M, K)).astype(np.float16)
    W = (rng.integers(0, 2 ** 30, size=(K // 10, N), dtype=np.int64)).astype(np.uint32).view(np.int32)
    G = (K + group - 1) // group
    s = np.abs(rng.standard_normal((G, N)) * 0.02).astype(np.float16) + np.float16(1e-3)
    z = (rng.standard_normal((G, N)) * 2).astype(np.float16) if zp else None
    return A, W, s, z


@pytest.fixture(params=["stream", "ring"])
def int3_kernel(request, cuda_device):
    """Both INT3 kernels: the register-streaming one (the default) and the
    warp-specialized TMA-ring one."""
    prev = t4_cuda_b200.set_int3_kernel(request.param)
    yield request.param
    t4_cuda_b200.set_int3_kernel(prev)
    assert t4_cuda_b200.device_error(cuda_device) == 0


@pytest.mark.parametrize("M,K,N,group,zp", [
    (1, 4100, 4096, 128, False),     # Llama K=4096 padded to a multiple of 10, group 128
    (1, 4100, 1024, 100, True),
    (1, 14340, 256, 128, False),
    (3, 260, 64, 128, True),         # words straddle group boundaries
    (9, 100, 60, 100, True),         # N % 4 != 0, two m-tiles
    (16, 200, 128, 32, False),
    (2, 10, 8, 100, True),           # one word row; K % 4 != 0 activation path
    (20, 1000, 72, 13, True),        # odd group size, M > 16
])
def test_int3_vs_oracle(cuda_device, int3_kernel, M, K, N, group, zp):
    rng = np.random.default_rng(abs(hash((M, K, N, group, zp))) % 2 ** 32)
    A, W, s, z = make_int3(rng, M, K, N, group, zp)
    zt = _dev(z, cuda_device) if zp else torch.empty(0, dtype=torch.float16, device=cuda_device)
    C = t4_kernels.fused_h17_gemv_s3(_dev(A, cuda_device), _dev(W, cuda_device), _dev(s, cuda_device), zt,
                                     group_size=group)
    assert_gemm_close(C, oracle.ref_int3_gemv(A, W, s, z, group), f"M={M} K={K} N={N} g={group} zp={zp}")


def test_one_dimensional_activation(cuda_device):
    """bindings.cpp:211-213: A of shape (K,) gives C of shape (1, N)."""
    rng = np.random.default_rng(4)
    A, W, s, z = make_int3(rng, 1, 200, 64, 100, True)
    C = t4_kernels.fused_h17_gemv_s3(_dev(A[0], cuda_device), _dev(W, cuda_device), _dev(s, cuda_device),
                                     _dev(z, cuda_device))
    assert C.shape == (1, 64)
    assert_gemm_close(C, oracle.ref_int3_gemv(A, W, s, z, 100))


def test_checks_mirror_the_reference(cuda_device):
    A = torch.zeros(1, 200, dtype=torch.float16, device=cuda_device)
    W = torch.zeros(20, 8, dtype=torch.int32, device=cuda_device)
    s = torch.ones(2, 8, dtype=torch.float16, device=cuda_device)
    with pytest.raises(RuntimeError, match="multiple of 10"):
        t4_kernels.fused_h17_gemv_s3(A[:, :195], W, s, s)
    with pytest.raises(RuntimeError, match="K/10"):
        t4_kernels.fused_h17_gemv_s3(A, W[:19], s, s)
    with pytest.raises(RuntimeError, match="num_groups"):
        t4_kernels.fused_h17_gemv_s3(A, W, s[:1], s[:1])
    with pytest.raises(RuntimeError, match="group_size"):
        t4_kernels.fused_h17_gemv_s3(A, W, torch.ones(29, 8, dtype=torch.float16, device=cuda_device), None,
                                     group_size=7)
    with pytest.raises(RuntimeError, match="contiguous"):
        t4_kernels.fused_h17_gemv_s3(A, W.t().contiguous().t(), s, s)


@pytest.mark.parametrize("group", [128, 100])
@pytest.mark.parametrize("K,N", [(4100, 4096), (4100, 14336), (14340, 4096), (14340, 14336)])
def test_int3_benchmark_configs(cuda_device, int3_kernel, K, N, group):
    """The INT3 configuration the benchmark reports (M = 1, K in {4096, 14336}
    padded to 4100 / 14340, N in {4096, 14336}) at full size on the GPU; the
    oracle checks a fixed random subset of columns (columns are independent):
    every 64-column block contributes two, plus the first and last."""
    rng = np.random.default_rng(K + N + group)
    A = rng.standard_normal((1, K), dtype=np.float32).astype(np.float16)
    W = rng.integers(0, 2 ** 30, size=(K // 10, N), dtype=np.uint32).view(np.int32)
    G = (K + group - 1) // group
    s = (np.abs(rng.standard_normal((G, N), dtype=np.float32)) * 0.02 + 1e-3).astype(np.float16)
    C = t4_kernels.fused_h17_gemv_s3(_dev(A, cuda_device), _dev(W, cuda_device), _dev(s, cuda_device),
                                     torch.empty(0, dtype=torch.float16, device=cuda_device), group_size=group)
    assert bool(torch.isfinite(C).all())
    cols = {0, N - 1}
    for b0 in range(0, N, 64):
        cols.update(rng.choice(np.arange(b0, min(N, b0 + 64)), size=2, replace=False).tolist())
    cols = np.array(sorted(cols))
    ref = oracle.ref_int3_gemv(A, W[:, cols], s[:, cols], None, group)
    y = C[:, torch.from_numpy(cols).to(cuda_device)]
    assert_gemm_close(y, ref, f"{int3_kernel}: K={K} N={N} g={group} ({len(cols)} columns checked)")
