"""Parity of the fused W4A16 GEMV / GEMM with the oracle.

Gate (the GEMM tolerance of this path's correctness contract, written here):
against the fp32-accumulated
product of fp16 activations and contract-dequantized fp16 weights,
    max |y - y_ref| <= 1e-2 * max |y_ref|      (max relative error)
    mean |y - y_ref| <= 1e-3 * mean |y_ref|    (mean absolute error)
plus the reference's own absolute gates on its own cases (0.5 in
tests/test_fused_gemm_correctness.py:38, 2.0 in harness/verify_fused_gemm.py:79).
"""

import hashlib
import json
import os

import numpy as np
import pytest
import torch

import oracle
import t4_cuda_b200
import t4_kernels
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu

MAX_REL = 1e-2
MAE_REL = 1e-3


def assert_gemm_close(C, ref, what=""):
    y = C.detach().float().cpu().numpy()
    assert y.shape == ref.shape, (y.shape, ref.shape)
    assert np.all(np.isfinite(y)), what
    err = np.abs(y - ref)
    max_rel = err.max() / max(np.abs(ref).max(), 1e-30)
    mae = err.mean() / max(np.abs(ref).mean(), 1e-30)
    assert max_rel <= MAX_REL, f"{what}: max rel err {max_rel:.3e}"
    assert mae <= MAE_REL, f"{what}: mean abs err {mae:.3e} of mean |y|"
    return max_rel, mae


def make_case(rng, M, K, N, group, zp, dev):
    """Synthetic inputs with the BASELINE distributions: A ~ N(0,1) fp16,
    full-range random words, scales |N(0, 0.02)| + 1e-3."""
    A = rng.standard_normal((M, K)).astype(np.float16)
    W = rng.integers(0, 2 ** 32, size=(K // 8, N), dtype=np.int64).astype(np.uint32).view(np.int32)
    G = 1 if group is None else K // group
    s = (np.abs(rng.standard_normal((G, N)) * 0.02) + 1e-3).astype(np.float16)
    if zp == "int":
        z = rng.integers(0, 16, size=(G, N)).astype(np.float16)
    elif zp == "frac":
        z = (rng.standard_normal((G, N)) * 3).astype(np.float16)
    else:
        z = None
    t = lambda x: None if x is None else torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    return A, W, s, z, t(A), t(W), t(s), t(z)


SHAPES = [
    # M, K, N, group, zp
    (1, 4096, 4096, 128, None),      # the headline decode shape
    (1, 4096, 1024, 128, None),
    (4, 4096, 1024, 128, None),
    (8, 1024, 512, 128, None),
    (16, 1024, 256, 128, None),
    (1, 14336, 256, 128, None),
    (1, 8, 4, None, "int"),          # reference "known small matrix"
    (1, 8, 1, None, "int"),          # reference "minimum K, single N"
    (2, 64, 60, None, "int"),        # N % 4 != 0: scalar load path
    (3, 256, 128, 64, "int"),
    (5, 520, 72, 8, "frac"),         # K % 32 != 0, group 8, fractional zero points
    (9, 96, 64, 32, None),           # two m-tiles
    (17, 256, 192, 128, "int"),      # M > 16: row chunks
    (33, 128, 64, None, None),
    (2, 1024, 200, None, "frac"),    # per-column scales, N tail inside a 16-column tile
    (3, 512, 520, 256, "int"),       # odd tile count, group of 32 word rows
    (2, 512, 14336, 64, "int"),      # 6-7 tiles per CTA (4 + 2/3 tile groups), 8-row flush blocks
    (12, 2048, 2720, 128, "frac"),   # M > 8: two batch tiles
    (1, 1024, 9600, 128, None),      # 4-5 tiles per CTA (a lone last tile)
    (3, 256, 7904, 128, "int"),      # 3-4 tiles per CTA (three-tile groups)
    (4, 1024, 512, 32, None),        # group 32: not the decode kernel's (falls back)
    (16, 4096, 2400, 128, "int"),    # M * K > 32768 with >= 148 column tiles: decode kernel, 4 ring stages
    (4, 14336, 2384, 128, "frac"),   # same at K = 14336 (57 KB of activations per batch row pair)
    (16, 4096, 1024, 128, None),     # M * K > 32768 with 64 tiles: the stream kernel's K split
]


@pytest.fixture(params=["auto", "stream", "generic"])
def gemv_kernel(request, cuda_device):
    prev = t4_cuda_b200.set_gemv_kernel(request.param)
    yield request.param
    t4_cuda_b200.set_gemv_kernel(prev)
    assert t4_cuda_b200.device_error(cuda_device) == 0


@pytest.mark.parametrize("signed", [True, False])
@pytest.mark.parametrize("M,K,N,group,zp", SHAPES)
def test_fused_gemm_vs_oracle(cuda_device, gemv_kernel, signed, M, K, N, group, zp):
    rng = np.random.default_rng(abs(hash((M, K, N, group, zp, signed))) % 2 ** 32)
    A, W, s, z, At, Wt, st, zt = make_case(rng, M, K, N, group, zp, cuda_device)
    op = t4_kernels.fused_w4a16_gemm_s4 if signed else t4_kernels.fused_w4a16_gemm_u4
    C = op(At, Wt, st if group else st.reshape(-1), zt)
    assert C.shape == (M, N) and C.dtype == torch.float16
    ref = oracle.ref_w4_gemm(A, W, s, z, signed=signed)
    assert_gemm_close(C, ref, f"{gemv_kernel}: M={M} K={K} N={N} g={group} zp={zp}")


@pytest.mark.parametrize("M,K,N", [(1, 4096, 4096), (1, 4096, 1024), (4, 4096, 14336), (1, 14336, 4096),
                                   (16, 2048, 512), (3, 1024, 4160)])
def test_streaming_kernel_matches_generic(cuda_device, M, K, N):
    """The two kernels see the same inputs; both pass the oracle gate and agree
    with each other far inside it.  Repeated calls are bit-identical (the
    split-tile fix-up sums in a fixed order)."""
    rng = np.random.default_rng(M * 7 + K + N)
    A, W, s, z, At, Wt, st, zt = make_case(rng, M, K, N, 128, None, cuda_device)
    prev = t4_cuda_b200.set_gemv_kernel("generic")
    try:
        Cg = t4_kernels.fused_w4a16_gemm_s4(At, Wt, st, None)
    finally:
        t4_cuda_b200.set_gemv_kernel(prev)
    Ca = t4_kernels.fused_w4a16_gemm_s4(At, Wt, st, None)
    Cb = t4_kernels.fused_w4a16_gemm_s4(At, Wt, st, None)
    assert torch.equal(Ca, Cb)
    ref = oracle.ref_w4_gemm(A, W, s, None, signed=True)
    assert_gemm_close(Ca, ref, "auto")
    assert_gemm_close(Cg, ref, "generic")
    d = (Ca.float() - Cg.float()).abs().max().item()
    assert d <= 2e-3 * np.abs(ref).max()
    assert t4_cuda_b200.device_error(cuda_device) == 0


def test_scale_shapes_agree(cuda_device):
    """(N,), (1, N) and (K/K, N) per-column scales are the same thing."""
    rng = np.random.default_rng(3)
    A, W, s, z, At, Wt, st, zt = make_case(rng, 2, 512, 128, None, "int", cuda_device)
    c1 = t4_kernels.fused_w4a16_gemm_s4(At, Wt, st, zt)
    c2 = t4_kernels.fused_w4a16_gemm_s4(At, Wt, st.reshape(-1), zt.reshape(-1))
    assert torch.equal(c1, c2)


def test_reference_cases(cuda_device):
    """The reference's own CPU results (tests/golden/gemm_cases.npz)."""
    d = np.load(os.path.join(GOLDEN, "gemm_cases.npz"))
    tags = sorted({k.rsplit("_", 1)[0] for k in d.files})
    for t in tags:
        signed = bool(d[t + "_signed"])
        op = t4_kernels.fused_w4a16_gemm_s4 if signed else t4_kernels.fused_w4a16_gemm_u4
        dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(cuda_device)
        C = op(dev(d[t + "_A"]), dev(d[t + "_W"]), dev(d[t + "_s"]), dev(d[t + "_z"]))
        # reference gate: max abs <= 0.5 against its fp16 result
        assert (C.float().cpu().numpy() - d[t + "_c16"].astype(np.float32)).__abs__().max() <= 0.5, t
        if np.abs(d[t + "_c32"]).max() > 0:
            assert_gemm_close(C, d[t + "_c32"], t)


def test_reference_seed42_harness_case(cuda_device):
    with open(os.path.join(GOLDEN, "gemm_seed42.json")) as f:
        ref = json.load(f)
    torch.manual_seed(42)
    A = torch.randn((1, 1024), dtype=torch.float16)
    W = torch.randint(0, 0x7FFFFFFF, (128, 1024), dtype=torch.int32)
    scale = torch.rand((1024,), dtype=torch.float16) * 0.1 + 0.05
    zero = torch.randint(0, 8, (1024,), dtype=torch.float16)
    h = hashlib.sha256()
    for a in (A.numpy(), W.numpy(), scale.numpy(), zero.numpy()):
        h.update(np.ascontiguousarray(a).tobytes())
    if h.hexdigest() != ref["input_sha256"]:
        pytest.skip("torch CPU generator differs from the one that made the fixture")
    for kind, op in (("u4", t4_kernels.fused_w4a16_gemm_u4), ("s4", t4_kernels.fused_w4a16_gemm_s4)):
        C = op(A.to(cuda_device), W.to(cuda_device), scale.to(cuda_device), zero.to(cuda_device))
        exp16 = np.asarray(ref[kind + "_c16"], np.uint16).view(np.float16).astype(np.float32)
        assert np.abs(C.float().cpu().numpy().reshape(-1) - exp16).max() < 2.0     # the harness gate
        assert_gemm_close(C, np.asarray(ref[kind + "_c32"], np.float32).reshape(1, -1), kind)


def test_sharded_columns_match_full(cuda_device):
    """A column slice of W (a shard) gives the same columns of C, bit for bit."""
    rng = np.random.default_rng(21)
    A, W, s, z, At, Wt, st, zt = make_case(rng, 4, 2048, 512, 128, None, cuda_device)
    full = t4_kernels.fused_w4a16_gemm_s4(At, Wt, st, None)
    part = t4_kernels.fused_w4a16_gemm_s4(At, Wt[:, 128:256].contiguous(), st[:, 128:256].contiguous(), None)
    assert torch.equal(full[:, 128:256], part)


def test_bad_shapes_raise(cuda_device):
    A = torch.zeros(1, 64, dtype=torch.float16, device=cuda_device)
    W = torch.zeros(8, 16, dtype=torch.int32, device=cuda_device)
    s = torch.ones(1, 16, dtype=torch.float16, device=cuda_device)
    with pytest.raises(RuntimeError):
        t4_kernels.fused_w4a16_gemm_u4(A[:, :60], W, s, None)            # K % 8
    with pytest.raises(RuntimeError):
        t4_kernels.fused_w4a16_gemm_u4(A, W[:7], s, None)                # W rows != K/8
    with pytest.raises(RuntimeError):
        t4_kernels.fused_w4a16_gemm_u4(A, W, torch.ones(3, 16, dtype=torch.float16, device=cuda_device), None)
    with pytest.raises(RuntimeError):
        t4_kernels.fused_w4a16_gemm_u4(A, W, s[:, :8], None)             # scale columns != N


def test_stream_kernel_inside_graph_capture(cuda_device):
    """A shape only the split-tile stream kernel takes (M * K too large for the
    decode kernel's resident activations, fewer tiles than SMs), first called
    while a brand-new stream is being captured: the kernel's workspace is made
    at capture time, and every replay equals the eager result bit for bit (the
    stream kernel reduces its split tiles in a fixed order)."""
    rng = np.random.default_rng(33)
    A, W, s, z, At, Wt, st, zt = make_case(rng, 16, 8192, 512, 128, None, cuda_device)
    eager = t4_kernels.fused_w4a16_gemm_s4(At, Wt, st, None)
    ref = oracle.ref_w4_gemm(A, W, s, None, signed=True)
    assert_gemm_close(eager, ref, "s4")
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=torch.cuda.Stream(cuda_device)):
        out = t4_kernels.fused_w4a16_gemm_s4(At, Wt, st, None)
    for _ in range(3):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
    assert t4_cuda_b200.device_error(cuda_device) == 0
