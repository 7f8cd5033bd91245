"""The allocation-free decode GEMV, t4b_fused_w4a16_gemv_noalloc, called through the C ABI.

Who needs it: callers that cannot allocate device memory while they run -- a
serving engine that reserves all of HBM for its own pool at start-up, or a host
runtime that forbids cudaMalloc once it is serving.  The regular matmul entry
points allocate a small workspace on their first call on a stream; this one
keeps its scratch in a fixed 4 MiB array inside the library instead.

What is checked:
  * on two calls in a row (different shapes, formats and zero points, both
    sharing the one scratch array, no synchronisation between them) its
    output matches the existing entry point's (t4b_fused_w4a16_gemm_s4 / _u4)
    and the oracle (oracle.ref_w4_gemm) within the GEMV tolerance used by the
    other parity tests:
        max |y - y_ref| <= 1e-2 * max |y_ref|,  mean |y - y_ref| <= 1e-3 * mean |y_ref|;
  * it made no workspace on the fresh stream it ran on (the existing entry
    point, as a control, does make one on its own fresh stream), and its error
    word is clear afterwards;
  * a shape too large for the array is refused with T4B_ERR_SCRATCH_LIMIT.

The file name makes pytest collect it last.  It passes on its own in a fresh
process (its first call looks up the array on the device) and after the rest.
"""

import ctypes

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

MAX_REL = 1e-2
MAE_REL = 1e-3
T4B_ERR_SCRATCH_LIMIT = 6


def _ptr(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _case(gen, M, K, N, group, zp, dev):
    A = torch.randn(M, K, generator=gen).half()
    W = torch.randint(-2 ** 31, 2 ** 31, (K // 8, N), generator=gen, dtype=torch.int64).to(torch.int32)
    S = (torch.randn(K // group, N, generator=gen).abs() * 0.02 + 1e-3).half()
    Z = torch.randint(0, 16, (K // group, N), generator=gen).half() if zp else None
    to = lambda t: None if t is None else t.to(dev)
    return to(A), to(W), to(S), to(Z)


def _noalloc(lib, case, M, N, K, group, signed, stream):
    A, W, S, Z = case
    C = torch.empty(M, N, dtype=torch.float16, device=A.device)
    st = lib.t4b_fused_w4a16_gemv_noalloc(_ptr(A), _ptr(W), _ptr(S), _ptr(Z), _ptr(C), M, N, K, group,
                                          1 if signed else 0, stream)
    assert st == 0, lib.t4b_status_string(st)
    return C


def _existing(lib, case, M, N, K, group, signed, stream):
    A, W, S, Z = case
    C = torch.empty(M, N, dtype=torch.float16, device=A.device)
    f = lib.t4b_fused_w4a16_gemm_s4 if signed else lib.t4b_fused_w4a16_gemm_u4
    st = f(_ptr(A), _ptr(W), _ptr(S), _ptr(Z), _ptr(C), M, N, K, group, stream)
    assert st == 0, lib.t4b_status_string(st)
    return C


def _assert_close(y, ref, what):
    y = y.float().cpu().numpy()
    ref = ref.float().cpu().numpy()
    assert np.all(np.isfinite(y)), what
    err = np.abs(y - ref)
    max_rel = err.max() / max(np.abs(ref).max(), 1e-30)
    mae = err.mean() / max(np.abs(ref).mean(), 1e-30)
    assert max_rel <= MAX_REL, f"{what}: max rel err {max_rel:.3e}"
    assert mae <= MAE_REL, f"{what}: mean abs err {mae:.3e}"


def _workspace_bytes(lib, stream):
    n = ctypes.c_size_t(0)
    assert lib.t4b_workspace_bytes(stream, ctypes.byref(n)) == 0
    return n.value


def test_noalloc_gemv_matches_existing_entry_point_on_two_calls_in_a_row(cuda_device):
    from t4_cuda_b200 import _lib
    lib = _lib.load()
    dev = cuda_device
    gen = torch.Generator().manual_seed(1234)
    # (M, K, N, group, signed, zero points): the decode shape, then a batched
    # unsigned case with zero points whose split tiles reuse the same scratch.
    shapes = [(1, 4096, 4096, 128, True, False), (16, 4096, 1024, 128, False, True)]
    cases = [_case(gen, M, K, N, g, zp, dev) for (M, K, N, g, _, zp) in shapes]
    torch.cuda.synchronize(dev)
    fresh = torch.cuda.Stream(dev)                   # no call of this library has used it
    s_fresh = ctypes.c_void_p(fresh.cuda_stream)
    assert _workspace_bytes(lib, s_fresh) == 0
    got = [_noalloc(lib, c, M, N, K, g, s, s_fresh) for c, (M, K, N, g, s, _) in zip(cases, shapes)]
    fresh.synchronize()
    assert _workspace_bytes(lib, s_fresh) == 0       # nothing was allocated for it
    err = ctypes.c_uint(1)
    assert lib.t4b_device_error(s_fresh, ctypes.byref(err), 0) == 0
    assert err.value == 0
    # control: the existing entry point on another fresh stream makes its workspace there
    other = torch.cuda.Stream(dev)
    s_other = ctypes.c_void_p(other.cuda_stream)
    want = [_existing(lib, c, M, N, K, g, s, s_other) for c, (M, K, N, g, s, _) in zip(cases, shapes)]
    other.synchronize()
    assert _workspace_bytes(lib, s_other) > 0
    for y, ref, (M, K, N, g, signed, zp), (A, W, S, Z) in zip(got, want, shapes, cases):
        _assert_close(y, ref, f"noalloc vs existing {(M, K, N, g, signed, zp)}")
        exact = oracle.ref_w4_gemm(A.cpu().numpy(), W.cpu().numpy(), S.cpu().numpy(),
                                   None if Z is None else Z.cpu().numpy(), signed=signed)
        _assert_close(y, torch.from_numpy(exact), f"noalloc vs oracle {(M, K, N, g, signed, zp)}")


def test_noalloc_gemv_refuses_shapes_beyond_its_scratch(cuda_device):
    from t4_cuda_b200 import _lib
    lib = _lib.load()
    dev = cuda_device
    M, K, N, g = 16, 4096, 128256, 128          # a vocabulary-sized projection at M = 16
    A = torch.zeros(M, K, dtype=torch.float16, device=dev)
    W = torch.zeros(K // 8, N, dtype=torch.int32, device=dev)
    S = torch.ones(K // g, N, dtype=torch.float16, device=dev)
    C = torch.empty(M, N, dtype=torch.float16, device=dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    st = lib.t4b_fused_w4a16_gemv_noalloc(_ptr(A), _ptr(W), _ptr(S), None, _ptr(C), M, N, K, g, 1, stream)
    assert st == T4B_ERR_SCRATCH_LIMIT
    assert b"scratch" in lib.t4b_status_string(st)
