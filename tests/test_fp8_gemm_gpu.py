"""The fused FP8-E4M3 weight GEMM (t4b_fused_w8a16_gemm_fp8) against the oracle.

* Every one of the 254 non-NaN E4M3 codes, through the GEMM with A = I: each
  output is one weight, fp16(e4m3 * s), and must equal the oracle's exactly
  (as a value: code 0x80, -0, comes out of the sum as +0).
* Random codes (no NaN) at decode and prefill shapes, per-column and grouped
  scales, within the GEMM gate used everywhere in these tests:
  max |y - y_ref| <= 1e-2 max |y_ref|, mean |y - y_ref| <= 1e-3 mean |y_ref|.
* A NaN weight poisons exactly its column.
"""

import numpy as np
import pytest
import torch

import oracle
import t4_cuda_b200
from tests.test_gemv_gpu import assert_gemm_close

pytestmark = pytest.mark.gpu


def _t(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


@pytest.mark.parametrize("scale_kind", ["one", "random"])
def test_every_code_exactly(cuda_device, scale_kind):
    K = N = 256
    codes = ((np.arange(K)[:, None] + 7 * np.arange(N)[None, :]) % 256).astype(np.uint8)
    # the two NaN codes would poison whole columns (0 * NaN in the identity
    # product); NaN gets its own test below
    codes[(codes & 0x7F) == 0x7F] = 0x00
    W = oracle.pack_fp8(codes)
    rng = np.random.default_rng(5)
    s = (np.ones((1, N)) if scale_kind == "one" else np.abs(rng.standard_normal((1, N))) * 0.5 + 0.01)
    s = s.astype(np.float16)
    A = np.eye(K, dtype=np.float16)
    C = t4_cuda_b200.fused_w8a16_gemm_fp8(_t(A, cuda_device), _t(W, cuda_device), _t(s, cuda_device))
    got = C.cpu().numpy()
    exp = oracle.dequant_fp8_matrix(W, s)
    assert not np.isnan(exp).any()
    # equal values (the sum turns the weight -0 of code 0x80 into +0, and
    # fp16 values are otherwise equal exactly when their bits are)
    assert np.array_equal(got, exp)
    assert t4_cuda_b200.device_error(cuda_device) == 0


def _random_case(rng, M, K, N, group):
    codes = rng.integers(0, 256, size=(K, N), dtype=np.int64).astype(np.uint8)
    codes[(codes & 0x7F) == 0x7F] = 0x3E          # no NaN codes
    W = oracle.pack_fp8(codes)
    G = 1 if group is None else K // group
    s = (np.abs(rng.standard_normal((G, N))) * 0.02 + 1e-3).astype(np.float16)
    A = rng.standard_normal((M, K)).astype(np.float16)
    return A, W, s


@pytest.mark.parametrize("M,K,N,group", [
    (1, 4096, 4096, 128),      # decode, K split over the SMs
    (1, 4096, 1024, 128),
    (4, 14336, 512, 128),
    (16, 1024, 768, None),     # per-column scales
    (64, 512, 1024, 64),
    (200, 2048, 520, 128),     # ragged M and N
    (512, 4096, 4096, 128),    # prefill
])
def test_fp8_gemm_vs_oracle(cuda_device, M, K, N, group):
    rng = np.random.default_rng(M * 7 + K + N)
    A, W, s = _random_case(rng, M, K, N, group)
    sc = s if group is not None else s.reshape(-1)
    C = t4_cuda_b200.fused_w8a16_gemm_fp8(_t(A, cuda_device), _t(W, cuda_device), _t(sc, cuda_device))
    torch.cuda.synchronize(cuda_device)
    assert t4_cuda_b200.device_error(cuda_device) == 0
    assert_gemm_close(C, oracle.ref_fp8_gemm(A, W, s), f"fp8 M={M} K={K} N={N} g={group}")


def test_nan_weight_poisons_its_column(cuda_device):
    rng = np.random.default_rng(3)
    A, W, s = _random_case(rng, 8, 256, 64, 128)
    codes = oracle.unpack_fp8_codes(W)
    codes[17, 5] = 0xFF
    W = oracle.pack_fp8(codes)
    C = t4_cuda_b200.fused_w8a16_gemm_fp8(_t(A, cuda_device), _t(W, cuda_device), _t(s, cuda_device)).float()
    assert bool(torch.isnan(C[:, 5]).all())
    assert bool(torch.isfinite(torch.cat([C[:, :5], C[:, 6:]], dim=1)).all())


def test_fp8_checks(cuda_device):
    A = torch.zeros(2, 128, dtype=torch.float16, device=cuda_device)
    W = torch.zeros(32, 64, dtype=torch.int32, device=cuda_device)
    s = torch.ones(64, dtype=torch.float16, device=cuda_device)
    with pytest.raises(RuntimeError, match="K/4"):
        t4_cuda_b200.fused_w8a16_gemm_fp8(A, W[:31], s)
    with pytest.raises(RuntimeError, match="FP16"):
        t4_cuda_b200.fused_w8a16_gemm_fp8(A.float(), W, s)
    with pytest.raises(RuntimeError, match="not supported"):      # group of 32 < the kernel's 64
        t4_cuda_b200.fused_w8a16_gemm_fp8(A, W, torch.ones(4, 64, dtype=torch.float16, device=cuda_device))
