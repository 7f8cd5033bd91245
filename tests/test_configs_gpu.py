"""Parity at every configuration the benchmark reports, checked against the oracle.

The shapes are the reference's own fused-GEMM shape list
(tests/test_fused_gemm_correctness.py:86-113) extended to the benchmark's
workloads:
  * decode skinny GEMM: the four Llama-3-8B projection shapes
    (K, N) in {(4096, 4096), (4096, 1024), (4096, 14336), (14336, 4096)} at
    M in {1, 4, 8, 16}, through the default dispatch, plus the M = 16 stream
    kernel shape replayed inside a CUDA graph;
  * prefill GEMM: the same four shapes at M in {512, 2048, 4096} under both
    tensor-core kernel choices ("auto" = CTA pairs past M = 128, "tc_single");
  * Llama-3-70B projections (hidden 8192, intermediate 28672) as one GPU and
    as an 8-way column shard see them, at M in {1, 16, 256, 4096}, including
    the split-K shapes at K = 28672.

The whole product runs on the GPU at full size.  Because output columns (and
rows) are independent, the oracle (oracle.ref_w4_gemm, the fp32 product of
fp16 activations and contract-dequantized weights) is evaluated on a fixed
random subset: every 128-row M tile contributes rows, every 64-column block
contributes columns, and the first and last row and column are always in.
Gate, as everywhere in these tests: max |y - y_ref| <= 1e-2 max |y_ref| and
mean |y - y_ref| <= 1e-3 mean |y_ref| over the checked entries; every output
of the full tensor must be finite.
"""

import numpy as np
import pytest
import torch

import oracle
import t4_cuda_b200
import t4_kernels
from tests.test_gemv_gpu import assert_gemm_close

pytestmark = pytest.mark.gpu

SHAPES_8B = [(4096, 4096), (4096, 1024), (4096, 14336), (14336, 4096)]


def make_inputs(seed, M, K, N, dev, zp=False):
    """BASELINE distributions: A ~ N(0, 1) fp16, full-range random int32 words,
    group-128 scales |N(0, 0.02)| + 1e-3, optional integer zero points."""
    rng = np.random.default_rng(seed)
    A = rng.standard_normal((M, K), dtype=np.float32).astype(np.float16)
    W = rng.integers(0, 2 ** 32, size=(K // 8, N), dtype=np.uint32).view(np.int32)
    s = (np.abs(rng.standard_normal((K // 128, N), dtype=np.float32) * 0.02) + 1e-3).astype(np.float16)
    z = rng.integers(0, 16, size=(K // 128, N)).astype(np.float16) if zp else None
    t = lambda x: None if x is None else torch.from_numpy(x).to(dev)
    return rng, (A, W, s, z), (t(A), t(W), t(s), t(z))


def subset(rng, n, block, per_block, full_below):
    """Indices to check along a dimension of size n: all of them when
    n <= full_below, else per_block random ones from every block plus 0, n-1."""
    if n <= full_below:
        return np.arange(n)
    idx = {0, n - 1}
    for b0 in range(0, n, block):
        hi = min(n, b0 + block)
        idx.update(rng.choice(np.arange(b0, hi), size=min(per_block, hi - b0), replace=False).tolist())
    return np.array(sorted(idx))


def check(C, host, rng, signed, what, full_rows=16, full_cols=1024):
    A, W, s, z = host
    M, N = C.shape
    assert bool(torch.isfinite(C).all()), f"{what}: non-finite outputs"
    rows = subset(rng, M, 128, 4, full_rows)
    cols = subset(rng, N, 64, 2, full_cols)
    ref = oracle.ref_w4_gemm(A[rows], W[:, cols], s[:, cols], None if z is None else z[:, cols], signed=signed)
    y = C[torch.from_numpy(rows).to(C.device)][:, torch.from_numpy(cols).to(C.device)]
    return assert_gemm_close(y, ref, f"{what} ({len(rows)} rows x {len(cols)} columns checked)")


@pytest.mark.parametrize("M", [1, 4, 8, 16])
@pytest.mark.parametrize("K,N", SHAPES_8B)
def test_decode_batch_configs(cuda_device, K, N, M):
    rng, host, (At, Wt, st, _) = make_inputs(1000 + M * 7 + K + N, M, K, N, cuda_device)
    C = t4_kernels.fused_w4a16_gemm_s4(At, Wt, st, None)
    torch.cuda.synchronize(cuda_device)
    assert t4_cuda_b200.device_error(cuda_device) == 0
    check(C, host, rng, True, f"decode M={M} K={K} N={N}", full_cols=4096)


def test_decode_stream_shape_in_graph(cuda_device):
    """M = 16 at 14336 x 4096 (the split-tile stream kernel), eager and replayed
    from a CUDA graph: both pass the oracle gate and agree bit for bit."""
    M, K, N = 16, 14336, 4096
    rng, host, (At, Wt, st, _) = make_inputs(77, M, K, N, cuda_device)
    eager = t4_kernels.fused_w4a16_gemm_s4(At, Wt, st, None)
    check(eager, host, rng, True, "stream eager", full_cols=4096)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=torch.cuda.Stream(cuda_device)):
        out = t4_kernels.fused_w4a16_gemm_s4(At, Wt, st, None)
    for _ in range(2):
        out.zero_()
        g.replay()
        torch.cuda.synchronize(cuda_device)
        assert torch.equal(out, eager)
    del g
    assert t4_cuda_b200.device_error(cuda_device) == 0


@pytest.fixture(params=["auto", "tc_single"])
def tc_kernel(request, cuda_device):
    prev = t4_cuda_b200.set_gemv_kernel(request.param)
    yield request.param
    t4_cuda_b200.set_gemv_kernel(prev)
    assert t4_cuda_b200.device_error(cuda_device) == 0


@pytest.mark.parametrize("M", [512, 2048, 4096])
@pytest.mark.parametrize("K,N", SHAPES_8B)
def test_prefill_configs(cuda_device, tc_kernel, K, N, M):
    rng, host, (At, Wt, st, _) = make_inputs(2000 + M + K * 3 + N, M, K, N, cuda_device)
    C = t4_kernels.fused_w4a16_gemm_s4(At, Wt, st, None)
    torch.cuda.synchronize(cuda_device)
    check(C, host, rng, True, f"{tc_kernel} prefill M={M} K={K} N={N}")


# Llama-3-70B layer projections: one GPU (full N) and the 8-way column shard
# (N / 8) of q (8192 x 8192), k/v (8192 x 1024), gate/up (8192 x 28672) and
# down (28672 x 8192).
SHAPES_70B = [
    # M, K, N
    (1, 8192, 8192), (1, 8192, 28672), (1, 28672, 8192), (1, 8192, 128), (1, 28672, 1024),
    (16, 8192, 28672), (16, 28672, 8192), (16, 8192, 3584), (16, 28672, 1024),
    (256, 8192, 1024), (256, 28672, 1024), (256, 28672, 8192), (256, 8192, 28672), (256, 8192, 3584),
    (4096, 8192, 8192), (4096, 28672, 8192), (4096, 8192, 1024), (4096, 8192, 3584),
]


@pytest.mark.parametrize("M,K,N", SHAPES_70B)
def test_llama70b_shard_configs(cuda_device, M, K, N):
    rng, host, (At, Wt, st, zt) = make_inputs(3000 + M + K + N, M, K, N, cuda_device, zp=(M == 256))
    op = t4_kernels.fused_w4a16_gemm_u4 if M == 256 else t4_kernels.fused_w4a16_gemm_s4
    C = op(At, Wt, st, zt)
    torch.cuda.synchronize(cuda_device)
    assert t4_cuda_b200.device_error(cuda_device) == 0
    check(C, host, rng, M != 256, f"70B M={M} K={K} N={N}")
