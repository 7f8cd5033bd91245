"""Parity of the tcgen05 prefill GEMMs (M > 16) with the oracle: the
single-CTA kernel (128 x 256 tiles) and the CTA-pair kernel (cta_group::2,
256 x 256 tiles per pair, taken for M > 128 under "auto").

Same gate as the GEMV tests (max |y - y_ref| <= 1e-2 max |y_ref|, mean
|y - y_ref| <= 1e-3 mean |y_ref|) against the fp32 product of fp16 activations
and contract-dequantized fp16 weights (oracle.ref_w4_gemm).  The shapes cover
ragged M and N (partial 128 x 256 tiles), group 64 / 128 / per-column scales,
integer and fractional zero points, and both nibble formats.
"""

import numpy as np
import pytest
import torch

import oracle
import t4_cuda_b200
import t4_kernels
from tests.test_gemv_gpu import assert_gemm_close, make_case

pytestmark = pytest.mark.gpu

SHAPES = [
    # M, K, N, group, zp
    (64, 512, 512, 128, None),
    (128, 1024, 768, 128, "int"),
    (200, 256, 520, 64, "frac"),       # N tail inside a 256-column tile, group 64
    (17, 256, 192, 128, "int"),        # smallest M the kernel takes
    (300, 8192, 1024, None, None),     # per-column scales (one group); K split 8 ways
    (512, 4096, 1024, 128, None),
    (1000, 1024, 4096, 128, "int"),    # ragged M
    (257, 512, 512, 64, "int"),        # second pair holds one valid row
    (129, 1024, 264, 128, None),       # smallest M on pairs; N tail of 8 columns
    (2048, 4096, 1024, 128, None),
    (128, 8256, 512, 64, "frac"),      # 129 K steps split 17 x 7 + 10
    (512, 14336, 1024, 128, "int"),    # K split 8 ways, zero points
    (512, 14336, 4096, 128, "int"),    # CTA pairs split K in two (112 K steps each), zero points
]


@pytest.fixture(params=["auto", "tc_single"])
def tc_kernel(request, cuda_device):
    prev = t4_cuda_b200.set_gemv_kernel(request.param)
    yield request.param
    t4_cuda_b200.set_gemv_kernel(prev)
    assert t4_cuda_b200.device_error(cuda_device) == 0


@pytest.mark.parametrize("signed", [True, False])
@pytest.mark.parametrize("M,K,N,group,zp", SHAPES)
def test_tc_gemm_vs_oracle(cuda_device, tc_kernel, signed, M, K, N, group, zp):
    rng = np.random.default_rng(M * 31 + K * 7 + N + (1 if signed else 0))
    A, W, s, z, At, Wt, st, zt = make_case(rng, M, K, N, group, zp, cuda_device)
    op = t4_kernels.fused_w4a16_gemm_s4 if signed else t4_kernels.fused_w4a16_gemm_u4
    C = op(At, Wt, st if group else st.reshape(-1), zt)
    assert C.shape == (M, N) and C.dtype == torch.float16
    ref = oracle.ref_w4_gemm(A, W, s, z, signed=signed)
    assert_gemm_close(C, ref, f"{tc_kernel}: M={M} K={K} N={N} g={group} zp={zp}")


def test_tc_gemm_matches_generic_kernel(cuda_device):
    """The tensor-core result and the register-streaming kernel's agree far
    inside the gate, and repeated tensor-core calls are bit-identical."""
    rng = np.random.default_rng(7)
    A, W, s, z, At, Wt, st, zt = make_case(rng, 256, 2048, 2048, 128, None, cuda_device)
    prev = t4_cuda_b200.set_gemv_kernel("generic")
    try:
        Cg = t4_kernels.fused_w4a16_gemm_s4(At, Wt, st, None)
    finally:
        t4_cuda_b200.set_gemv_kernel(prev)
    C1 = t4_kernels.fused_w4a16_gemm_s4(At, Wt, st, None)
    C2 = t4_kernels.fused_w4a16_gemm_s4(At, Wt, st, None)
    assert torch.equal(C1, C2)
    d = (C1.float() - Cg.float()).abs().max().item()
    assert d <= 2e-3 * Cg.float().abs().max().item()


def test_pair_and_single_cta_kernels_agree(cuda_device):
    """Both tensor-core kernels accumulate each output in fp32 over K in the
    same 16-wide steps; their results agree far inside the gate.  (A shape
    with enough tiles that neither splits K.)"""
    rng = np.random.default_rng(8)
    A, W, s, z, At, Wt, st, zt = make_case(rng, 640, 2048, 8192, 128, "int", cuda_device)
    prev = t4_cuda_b200.set_gemv_kernel("tc_single")
    try:
        C1 = t4_kernels.fused_w4a16_gemm_u4(At, Wt, st, zt)
    finally:
        t4_cuda_b200.set_gemv_kernel(prev)
    C2 = t4_kernels.fused_w4a16_gemm_u4(At, Wt, st, zt)
    torch.cuda.synchronize(cuda_device)
    assert t4_cuda_b200.device_error(cuda_device) == 0
    d = (C1.float() - C2.float()).abs().max().item()
    assert d <= 1e-3 * C1.float().abs().max().item()


def test_split_k_matches_unsplit(cuda_device):
    """A shape with few tiles splits K across CTAs (partials summed in split
    order by the tile's last CTA); it agrees with the same product computed
    unsplit, as extra rows of a larger M, far inside the gate."""
    rng = np.random.default_rng(9)
    A, W, s, z, At, Wt, st, zt = make_case(rng, 256, 8192, 1024, 128, None, cuda_device)
    C = t4_kernels.fused_w4a16_gemm_s4(At, Wt, st, None)               # 8 tiles: K split 8 ways
    big = torch.cat([At] * 20)                                          # 5120 rows: 160 tiles, no split
    Cb = t4_kernels.fused_w4a16_gemm_s4(big, Wt, st, None)
    torch.cuda.synchronize(cuda_device)
    assert t4_cuda_b200.device_error(cuda_device) == 0
    d = (C.float() - Cb[:256].float()).abs().max().item()
    assert d <= 1e-3 * Cb.float().abs().max().item()
    assert torch.equal(C, t4_kernels.fused_w4a16_gemm_s4(At, Wt, st, None))   # deterministic
