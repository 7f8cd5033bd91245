"""Back-to-back dependent launches: every kernel here launches with
programmatic dependent launch (it may start while the previous kernel in the
stream still runs) and must read its activations and write its output only
after griddepcontrol.wait.  Each case chains two calls where the second one's
activations ARE the first one's output buffer (no kernel between them), runs
the chain eagerly and as a CUDA graph replayed with new inputs, and checks both
outputs against the oracle (the second fed the first's actual output), with
the usual gate (max rel err <= 1e-2 of max|y|, mean abs err <= 1e-3 of mean|y|)."""

import numpy as np
import pytest
import torch

import oracle
import t4_cuda_b200
import t4_kernels
from tests.test_gemv_gpu import assert_gemm_close

pytestmark = pytest.mark.gpu


def _t(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def _w4(rng, K, N, dev, scale=0.02):
    W = rng.integers(0, 2 ** 32, size=(K // 8, N), dtype=np.int64).astype(np.uint32).view(np.int32)
    s = (np.abs(rng.standard_normal((K // 128, N))) * scale + 1e-3).astype(np.float16)
    return W, s, _t(W, dev), _t(s, dev)


def _run_chain(dev, first, second, x_np, ref_first, ref_second):
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        x = _t(x_np, dev)
        for _ in range(3):
            y = first(x)
            out = second(y)
        stream.synchronize()
        assert_gemm_close(y, ref_first(x_np), "first call, eager")
        assert_gemm_close(out, ref_second(y.cpu().numpy()), "chained call, eager")
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            y_g = first(x)
            out_g = second(y_g)
        rng = np.random.default_rng(17)
        for _ in range(3):
            xn = rng.standard_normal(x_np.shape).astype(np.float16)
            x.copy_(_t(xn, dev))
            g.replay()
            stream.synchronize()
            assert_gemm_close(y_g, ref_first(xn), "first call, graph")
            assert_gemm_close(out_g, ref_second(y_g.cpu().numpy()), "chained call, graph")
        del g
    assert t4_cuda_b200.device_error(dev) == 0


@pytest.mark.parametrize("M,K,N1,N2", [
    (1, 4096, 4096, 1024),      # decode GEMV -> decode GEMV
    (64, 1024, 1024, 512),      # single-CTA tcgen05 -> single-CTA
    (512, 4096, 1024, 4096),    # K split in a cluster -> CTA pairs
    (300, 2048, 2048, 768),     # CTA pairs -> CTA pairs (ragged M)
    (512, 14336, 4096, 512),    # pairs splitting K through the workspace -> K split in a cluster
])
def test_w4_chain(cuda_device, M, K, N1, N2):
    rng = np.random.default_rng(M + K + N1)
    x = rng.standard_normal((M, K)).astype(np.float16)
    W1, s1, W1t, s1t = _w4(rng, K, N1, cuda_device, scale=0.02 / np.sqrt(K / 1024))
    W2, s2, W2t, s2t = _w4(rng, N1, N2, cuda_device)
    _run_chain(cuda_device,
               lambda a: t4_kernels.fused_w4a16_gemm_s4(a, W1t, s1t, None),
               lambda a: t4_kernels.fused_w4a16_gemm_s4(a, W2t, s2t, None),
               x,
               lambda a: oracle.ref_w4_gemm(a, W1, s1, None, signed=True),
               lambda a: oracle.ref_w4_gemm(a, W2, s2, None, signed=True))


@pytest.mark.parametrize("M", [1, 64, 300])
def test_int3_chain(cuda_device, M):
    rng = np.random.default_rng(M)
    K1, N1, N2, g = 4100, 4000, 512, 128
    x = rng.standard_normal((M, K1)).astype(np.float16)
    W1 = rng.integers(0, 2 ** 30, size=(K1 // 10, N1), dtype=np.int64).astype(np.uint32).view(np.int32)
    s1 = (np.abs(rng.standard_normal((-(-K1 // g), N1))) * 0.01 + 1e-3).astype(np.float16)
    W2 = rng.integers(0, 2 ** 30, size=(N1 // 10, N2), dtype=np.int64).astype(np.uint32).view(np.int32)
    s2 = (np.abs(rng.standard_normal((-(-N1 // g), N2))) * 0.02 + 1e-3).astype(np.float16)
    W1t, s1t, W2t, s2t = _t(W1, cuda_device), _t(s1, cuda_device), _t(W2, cuda_device), _t(s2, cuda_device)
    Z = torch.empty(0, dtype=torch.float16, device=cuda_device)
    _run_chain(cuda_device,
               lambda a: t4_kernels.fused_h17_gemv_s3(a, W1t, s1t, Z, group_size=g),
               lambda a: t4_kernels.fused_h17_gemv_s3(a, W2t, s2t, Z, group_size=g),
               x,
               lambda a: oracle.ref_int3_gemv(a, W1, s1, None, g),
               lambda a: oracle.ref_int3_gemv(a, W2, s2, None, g))


@pytest.mark.parametrize("M", [1, 256])
def test_fp8_chain(cuda_device, M):
    rng = np.random.default_rng(M + 5)
    K, N1, N2 = 2048, 2048, 1024
    x = rng.standard_normal((M, K)).astype(np.float16)

    def make(Kx, Nx, scale):
        codes = rng.integers(0, 256, size=(Kx, Nx), dtype=np.int64).astype(np.uint8)
        codes[(codes & 0x7F) == 0x7F] = 0          # no NaN codes
        s = (np.abs(rng.standard_normal((Kx // 128, Nx))) * scale + 1e-3).astype(np.float16)
        return oracle.pack_fp8(codes), s

    W1, s1 = make(K, N1, 0.002)
    W2, s2 = make(N1, N2, 0.01)
    W1t, s1t, W2t, s2t = _t(W1, cuda_device), _t(s1, cuda_device), _t(W2, cuda_device), _t(s2, cuda_device)
    _run_chain(cuda_device,
               lambda a: t4_cuda_b200.fused_w8a16_gemm_fp8(a, W1t, s1t),
               lambda a: t4_cuda_b200.fused_w8a16_gemm_fp8(a, W2t, s2t),
               x,
               lambda a: oracle.ref_fp8_gemm(a, W1, s1),
               lambda a: oracle.ref_fp8_gemm(a, W2, s2))
