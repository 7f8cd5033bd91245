"""Host-side behaviour of the torch-facing ops that needs no GPU: the
reference rejects CPU tensors with RuntimeError (bindings.cpp:13-16 etc.) and
so must the drop-in; the repo-root ``t4_kernels`` module exposes the seven ops."""

import pytest
import torch

import t4_kernels
import t4_cuda_b200


OPS = ["dequantize_u4", "dequantize_s4", "dequantize_s3", "dequantize_fp8",
       "fused_w4a16_gemm_u4", "fused_w4a16_gemm_s4", "fused_h17_gemv_s3"]


def test_drop_in_module_exposes_the_reference_names():
    # tests/run_all_cuda_tests.py:76-77 checks exactly these attributes
    for name in OPS:
        assert callable(getattr(t4_kernels, name))
        assert getattr(t4_kernels, name) is getattr(t4_cuda_b200, name)


def test_cpu_tensors_are_rejected_like_the_reference():
    w = torch.zeros(4, dtype=torch.int32)
    s = torch.ones(4, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        t4_kernels.dequantize_u4(w, s, s)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        t4_kernels.dequantize_fp8(w, s)
    A = torch.zeros(1, 8, dtype=torch.float16)
    W = torch.zeros(1, 4, dtype=torch.int32)
    sc = torch.ones(1, 4, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        t4_kernels.fused_w4a16_gemm_s4(A, W, sc, sc)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        t4_kernels.fused_h17_gemv_s3(torch.zeros(10, dtype=torch.float16), torch.zeros(1, 4, dtype=torch.int32),
                                     sc, sc)


def test_mode_names():
    from t4_cuda_b200 import _lib
    assert _lib.MODES == {"contract": 0, "magic": 1}
