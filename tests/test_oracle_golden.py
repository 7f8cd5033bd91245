"""Pin the numpy oracle against golden vectors produced by the reference's own
CPU functions (tests/golden/make_golden.py).  CPU only."""

import hashlib
import json
import os

import numpy as np
import pytest
import torch

import oracle
from tests.conftest import GOLDEN


def _kats():
    with open(os.path.join(GOLDEN, "dequant_kats.json")) as f:
        return json.load(f)["cases"]


def _same_bits(got16, exp_bits):
    """Bit equality of fp16 arrays, every NaN counting as equal to every NaN."""
    g = np.asarray(got16, np.float16).reshape(-1)
    e = np.asarray(exp_bits, np.uint16).view(np.float16).reshape(-1)
    both_nan = np.isnan(g) & np.isnan(e)
    return np.all((g.view(np.uint16) == e.view(np.uint16)) | both_nan)


@pytest.mark.parametrize("case", _kats(), ids=lambda c: c["name"])
def test_dequant_contract_matches_reference_cpu(case):
    s = np.asarray(case["scales_f16"], np.uint16).view(np.float16)
    if case["kind"] == "fp8":
        got = oracle.dequantize_fp8(case["words"], s, mode="contract")
        valid = np.repeat(np.asarray(case["valid"], bool).reshape(-1, 4), 1, axis=0).reshape(-1)
        exp = np.asarray(case["expected_f16"], np.uint16)
        assert _same_bits(got[valid], exp[valid])
        return
    z = np.asarray(case["zeros_f16"], np.uint16).view(np.float16)
    got = oracle.dequantize(case["kind"], case["words"], s, z, mode="contract")
    assert _same_bits(got, case["expected_f16"]), case["source"]


def test_dequant_fuzz_u4_matches_reference_cpu():
    d = np.load(os.path.join(GOLDEN, "dequant_fuzz_u4.npz"))
    got = oracle.dequantize("u4", d["words"], d["scales"], d["zeros"], mode="contract")
    assert _same_bits(got, d["expected"].view(np.uint16))


def test_harness_kat_answers():
    """The printed answers of results/t4_colab_runtime_logs/02_verify_dequant.log:50-59."""
    u = oracle.dequantize("u4", [0xA7C13E59], [0.25], [2.0])
    assert u.tolist() == [1.75, 0.75, 3.0, 0.25, -0.25, 2.5, 1.25, 2.0]
    s = oracle.dequantize("s4", [0xF817E29A], [0.5], [0.0])
    assert s.tolist() == [-3.0, -3.5, 1.0, -1.0, 3.5, 0.5, -4.0, -0.5]


def test_magic_constants_are_exact():
    """harness/verify_dequant.py:47-83: 0x6400|u == 1024+u, 0x6400|(u^8) == 1032+s4."""
    for u in range(16):
        assert np.uint16(0x6400 | u).view(np.float16) == 1024 + u
        s4 = u - 16 if u >= 8 else u
        assert np.uint16(0x6400 | (u ^ 8)).view(np.float16) == 1032 + s4
    for e in range(8):
        s3 = e - 8 if e >= 4 else e
        assert np.uint16(0x6400 | (e ^ 4)).view(np.float16) == 1028 + s3


def test_magic_equals_contract_on_reference_kats():
    """The reference GPU kernels (magic arithmetic) matched its CPU oracle exactly
    on these words (results/t4_verify_20260801_091508.log:197-221, PASS rows)."""
    for w, s, z, kind in [(0x76543210, 1.0, 0.0, "u4"), (0x76543210, 0.5, 1.0, "u4"), (0x76543210, 0.5, 1.0, "s4"),
                          (0x00000000, 1.0, 0.0, "s4"), (0xA7C13E59, 0.25, 2.0, "u4")]:
        a = oracle.dequantize(kind, [w], [s], [z], mode="magic")
        b = oracle.dequantize(kind, [w], [s], [z], mode="contract")
        assert a.view(np.uint16).tolist() == b.view(np.uint16).tolist()


def test_magic_differs_where_reference_gpu_failed():
    """The reference GPU failed the 65000-scale edge (inf) and the randn*5 fuzz
    (max err 7.25) against its CPU oracle; the magic oracle reproduces both."""
    a = oracle.dequantize("u4", [0x76543210], [65000.0], [0.0], mode="magic")
    assert np.all(np.isinf(a))
    d = np.load(os.path.join(GOLDEN, "dequant_fuzz_u4.npz"))
    m = oracle.dequantize("u4", d["words"], d["scales"], d["zeros"], mode="magic").astype(np.float64)
    c = oracle.dequantize("u4", d["words"], d["scales"], d["zeros"], mode="contract").astype(np.float64)
    err = np.nanmax(np.abs(m - c)[np.isfinite(m) & np.isfinite(c)])
    assert 1.0 < err < 64.0


def test_gemm_oracle_matches_reference_cpu():
    d = np.load(os.path.join(GOLDEN, "gemm_cases.npz"))
    tags = sorted({k.rsplit("_", 1)[0] for k in d.files})
    assert tags
    for t in tags:
        signed = bool(d[t + "_signed"])
        got = oracle.ref_w4_gemm(d[t + "_A"], d[t + "_W"], d[t + "_s"], d[t + "_z"], signed=signed)
        exp = d[t + "_c32"]
        scale = max(1e-6, float(np.abs(exp).max()))
        assert np.abs(got - exp).max() <= 1e-5 * scale, t
        # the reference returns .half(); agree to one fp16 rounding
        assert np.abs(got.astype(np.float16).astype(np.float32) - d[t + "_c16"].astype(np.float32)).max() \
            <= 1e-3 * scale + 1e-6, t


def test_gemm_seed42_case():
    """harness/verify_fused_gemm.py:58-91 recipe (seed 42, M=1, K=N=1024)."""
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
    for kind, signed in (("u4", False), ("s4", True)):
        got = oracle.ref_w4_gemm(A.numpy(), W.numpy(), scale.numpy(), zero.numpy(), signed=signed).reshape(-1)
        exp = np.asarray(ref[kind + "_c32"], np.float32)
        assert np.abs(got - exp).max() <= 1e-5 * np.abs(exp).max()


def test_int3_oracle_matches_reference_cpu():
    d = np.load(os.path.join(GOLDEN, "int3_cases.npz"))
    for t in ("gate", "g128", "nozp"):
        g = int(d[t + "_group"])
        got = oracle.ref_int3_gemv(d[t + "_A"].astype(np.float16), d[t + "_W"], d[t + "_s"], d[t + "_z"],
                                   group_size=g)
        exp = d[t + "_c"]
        assert np.abs(got - exp).max() <= 1e-5 * np.abs(exp).max() + 1e-6, t


def test_int3_packer_roundtrip():
    rng = np.random.default_rng(0)
    q = rng.integers(0, 8, size=(16, 40))
    words = oracle.pack_int3(q)
    tc = oracle.unpack_int3_matrix(words.view(np.int32))
    assert np.array_equal(tc.T, np.where(q >= 4, q - 8, q))


def test_int4_packer_roundtrip():
    rng = np.random.default_rng(1)
    q = rng.integers(-8, 8, size=(64, 24))
    w = oracle.pack_int4(q)
    assert np.array_equal(oracle.gemm.unpack_w4_matrix(w, signed=True), q)
    # the word layout of tests/test_fused_gemm_correctness.py:11-15 (row 8kw+j = nibble j)
    wu = oracle.as_u32(w)
    assert ((wu[2, 5] >> 12) & 0xF) == (q[8 * 2 + 3, 5] & 0xF)


def test_fp8_oracle_matches_torch_e4m3fn():
    """The FP8 GEMM oracle decodes all 256 E4M3 codes as torch.float8_e4m3fn
    does (subnormals, NaN), and packs / unpacks bytes in K order."""
    import torch
    codes = np.arange(256, dtype=np.uint8)
    mine = oracle.e4m3_to_float(codes)
    ref = torch.from_numpy(codes).view(torch.float8_e4m3fn).double().numpy()
    assert np.array_equal(np.isnan(mine), np.isnan(ref))
    assert np.array_equal(mine[~np.isnan(mine)], ref[~np.isnan(ref)])
    rng = np.random.default_rng(0)
    c = rng.integers(0, 256, size=(64, 9), dtype=np.int64).astype(np.uint8)
    assert np.array_equal(oracle.unpack_fp8_codes(oracle.pack_fp8(c)), c)
    w = oracle.pack_fp8(c)
    assert (w.view(np.uint32)[3, 2] & 0xFF) == c[12, 2] and (w.view(np.uint32)[3, 2] >> 24) == c[15, 2]
