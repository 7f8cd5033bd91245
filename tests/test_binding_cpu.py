"""The torch binding of the fused W4A16 ops (t4_cuda_b200/bind/torch_ops.cpp):
it is built in-tree, loads, is wired to the loaded C library, and rejects bad
arguments with the same messages as the Python path (CPU tensors only here --
no kernel runs)."""

import pytest
import torch

from t4_cuda_b200 import ops


def test_binding_is_built_and_initialised():
    b = ops._binding()
    assert b is not None, "t4_cuda_b200/_torch_ops*.so is not built (python -m t4_cuda_b200.build)"
    for name in ("init", "fused_w4a16_gemm_u4", "fused_w4a16_gemm_s4", "fused_w4a16_gemm_grouped"):
        assert hasattr(b, name)


@pytest.mark.parametrize("op", ["t4b_fused_w4a16_gemm_u4", "t4b_fused_w4a16_gemm_s4"])
def test_cpu_tensors_rejected_like_the_python_path(op):
    b = ops._binding()
    fn = getattr(b, op[len("t4b_"):])
    A = torch.zeros(1, 64, dtype=torch.float16)
    W = torch.zeros(8, 16, dtype=torch.int32)
    S = torch.zeros(16, dtype=torch.float16)
    with pytest.raises(RuntimeError) as e_bind:
        fn(A, W, S, None)
    with pytest.raises(RuntimeError) as e_py:
        ops._fused(op, A, W, S, None)
    assert str(e_bind.value) == str(e_py.value) == "A must be a CUDA tensor"


def test_grouped_rejects_like_the_python_path():
    b = ops._binding()
    A = torch.zeros(1, 64, dtype=torch.float16)
    W = torch.zeros(8, 16, dtype=torch.int32)
    S = torch.zeros(16, dtype=torch.float16)
    cases = [
        ((A, [W, W], [S, S], None), "A must be a CUDA tensor"),
        ((A, [W, W], [S], None), "W_packed, scales and zero_points lists must have the same length"),
        ((A, [], [], None), "a grouped call takes 1 to 4 projections, got 0"),
        ((A, [W] * 5, [S] * 5, None), "a grouped call takes 1 to 4 projections, got 5"),
    ]
    for args, msg in cases:
        with pytest.raises(RuntimeError) as e_bind:
            b.fused_w4a16_gemm_grouped(*args, True)
        with pytest.raises(RuntimeError) as e_py:
            ops._fused_grouped(*args, True)
        assert str(e_bind.value) == str(e_py.value) == msg
