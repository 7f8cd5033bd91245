"""The torch binding of the fused W4A16 ops against the Python (ctypes) path:
the same kernels run, so outputs are bit-identical, and every argument check
raises the same RuntimeError message (the reference's checks,
src/bindings.cpp:64-132)."""

import numpy as np
import pytest
import torch

import oracle
from t4_cuda_b200 import ops
from tests.test_gemv_gpu import assert_gemm_close, make_case

pytestmark = pytest.mark.gpu

OPS = ["t4b_fused_w4a16_gemm_u4", "t4b_fused_w4a16_gemm_s4"]


@pytest.mark.parametrize("op", OPS)
@pytest.mark.parametrize("M,K,N,group,zp", [
    (1, 4096, 4096, 128, None),
    (1, 4096, 1024, 128, "int"),
    (4, 1024, 512, 64, "frac"),
    (16, 4096, 2400, 128, None),
    (64, 512, 512, 128, "int"),        # tcgen05 GEMM
    (2, 64, 60, None, "int"),          # per-column scales, N % 4 != 0
])
def test_binding_matches_python_path(cuda_device, op, M, K, N, group, zp):
    rng = np.random.default_rng(M * 7 + K + N)
    A, W, s, z, At, Wt, st, zt = make_case(rng, M, K, N, group, zp, cuda_device)
    b = ops._binding()
    assert b is not None
    S_arg = st if group else st.reshape(-1)
    C_bind = getattr(b, op[len("t4b_"):])(At, Wt, S_arg, zt)
    C_py = ops._fused(op, At, Wt, S_arg, zt)
    assert torch.equal(C_bind, C_py)
    assert_gemm_close(C_bind, oracle.ref_w4_gemm(A, W, s, z, signed=op.endswith("s4")), op)


def _bad_cases(dev):
    A = torch.zeros(2, 64, dtype=torch.float16, device=dev)
    W = torch.zeros(8, 16, dtype=torch.int32, device=dev)
    S = torch.ones(16, dtype=torch.float16, device=dev)
    return [
        (A.float(), W, S, None),                                   # A must be FP16
        (A, W.float(), S, None),                                   # W_packed must be Int32
        (A, W, S.float(), None),                                   # scales must be FP16
        (A[0], W, S, None),                                        # A must be 2-D
        (A, W[0], S, None),                                        # W_packed must be 2-D
        (A[:, :60], W, S, None),                                   # K % 8
        (A[:, :56], W, S, None),                                   # W_packed rows != K/8
        (A, W, S[:8], None),                                       # scales (N,) size
        (A, W, S.reshape(1, 16).expand(3, 16).contiguous(), None),  # groups must divide K
        (A, W, S.reshape(1, 16).expand(16, 16).contiguous(), None),  # group size K/16=4 not a multiple of 8
        (A, W, S, S.float()),                                      # zero_points must be FP16
        (A, W, S, torch.ones(2, 16, dtype=torch.float16, device=dev)),  # zero_points shape differs
        (torch.zeros(0, 64, dtype=torch.float16, device=dev), W, S, None),  # M = 0
    ]


@pytest.mark.parametrize("op", OPS)
def test_binding_errors_match_python_path(cuda_device, op):
    b = ops._binding()
    fn = getattr(b, op[len("t4b_"):])
    for i, args in enumerate(_bad_cases(cuda_device)):
        with pytest.raises(RuntimeError) as e_bind:
            fn(*args)
        with pytest.raises(RuntimeError) as e_py:
            ops._fused(op, *args)
        assert str(e_bind.value) == str(e_py.value), (i, str(e_bind.value), str(e_py.value))
