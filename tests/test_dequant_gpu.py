"""Parity of the flat dequantization kernels with the oracle: bit-exact in both
modes, on the reference's golden vectors and on seeded random inputs, through
the public ops (which call the C ABI)."""

import json
import os

import numpy as np
import pytest
import torch

import oracle
import t4_kernels
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu

OPS = {"u4": t4_kernels.dequantize_u4, "s4": t4_kernels.dequantize_s4, "s3": t4_kernels.dequantize_s3}


def assert_bits(got_t, exp16, mask=None):
    g = got_t.detach().cpu().numpy().astype(np.float16).reshape(-1)
    e = np.asarray(exp16, np.float16).reshape(-1)
    assert g.shape == e.shape
    if mask is not None:
        g, e = g[mask], e[mask]
    same = (g.view(np.uint16) == e.view(np.uint16)) | (np.isnan(g) & np.isnan(e))
    bad = np.flatnonzero(~same)
    assert bad.size == 0, f"{bad.size} mismatches, first at {bad[:5]}: got {g[bad[:5]]} expected {e[bad[:5]]}"


def words_t(words, dev):
    return torch.tensor(np.asarray(words, np.int64) & 0xFFFFFFFF, dtype=torch.int64).to(torch.int32).to(dev)


def f16_t(bits, dev):
    return torch.from_numpy(np.asarray(bits, np.uint16).view(np.float16).copy()).to(dev)


def _kats():
    with open(os.path.join(GOLDEN, "dequant_kats.json")) as f:
        return json.load(f)["cases"]


@pytest.mark.parametrize("case", _kats(), ids=lambda c: c["name"])
def test_reference_kats_contract(cuda_device, case):
    w = words_t(case["words"], cuda_device)
    s = f16_t(case["scales_f16"], cuda_device)
    if case["kind"] == "fp8":
        out = t4_kernels.dequantize_fp8(w, s)
        assert_bits(out, np.asarray(case["expected_f16"], np.uint16).view(np.float16),
                    mask=np.asarray(case["valid"], bool))
        return
    z = f16_t(case["zeros_f16"], cuda_device)
    out = OPS[case["kind"]](w, s, z)
    assert_bits(out, np.asarray(case["expected_f16"], np.uint16).view(np.float16))


def test_reference_fuzz_u4(cuda_device):
    d = np.load(os.path.join(GOLDEN, "dequant_fuzz_u4.npz"))
    out = t4_kernels.dequantize_u4(torch.from_numpy(d["words"]).to(cuda_device),
                                   torch.from_numpy(d["scales"]).to(cuda_device),
                                   torch.from_numpy(d["zeros"]).to(cuda_device))
    assert_bits(out, d["expected"])


def _random_inputs(rng, n, zkind):
    words = rng.integers(0, 2 ** 32, size=n, dtype=np.int64)
    s = (rng.standard_normal(n) * rng.choice([0.02, 1.0, 5.0])).astype(np.float16)
    if zkind == "zero":
        z = np.zeros(n, np.float16)
    elif zkind == "int":
        z = rng.integers(-16, 17, size=n).astype(np.float16)
    else:   # arbitrary fp16 values, including tiny ones that make q - z inexact in fp32
        z = (rng.standard_normal(n) * rng.choice([1e-4, 0.3, 5.0, 3000.0], size=n)).astype(np.float16)
    return words, s, z


@pytest.mark.parametrize("kind", ["u4", "s4", "s3"])
@pytest.mark.parametrize("mode", ["contract", "magic"])
@pytest.mark.parametrize("zkind", ["zero", "int", "any"])
@pytest.mark.parametrize("n", [1, 3, 4, 5, 1000, 4099])
def test_random_bit_exact(cuda_device, kind, mode, zkind, n):
    rng = np.random.default_rng(hash((kind, mode, zkind, n)) % 2 ** 32)
    words, s, z = _random_inputs(rng, n, zkind)
    if kind == "s3":
        words &= 0x3FFFFFFF
    out = OPS[kind](words_t(words, cuda_device), torch.from_numpy(s).to(cuda_device),
                    torch.from_numpy(z).to(cuda_device), mode=mode)
    assert out.shape == (n * (10 if kind == "s3" else 8),)
    assert_bits(out, oracle.dequantize(kind, words, s, z, mode=mode))


@pytest.mark.parametrize("mode", ["contract", "magic"])
def test_fp8_all_bytes_and_random(cuda_device, mode):
    rng = np.random.default_rng(5)
    words = np.concatenate([np.arange(0, 256, 4, dtype=np.int64) * 0x01010101 + 0x03020100,
                            rng.integers(0, 2 ** 32, size=2001, dtype=np.int64)])
    s = (rng.standard_normal(words.size) * 3).astype(np.float16)
    out = t4_kernels.dequantize_fp8(words_t(words, cuda_device), torch.from_numpy(s).to(cuda_device), mode=mode)
    assert_bits(out, oracle.dequantize_fp8(words, s, mode=mode))


@pytest.mark.parametrize("kind", ["u4", "s4", "s3"])
def test_broadcast_and_missing_zero_point(cuda_device, kind):
    rng = np.random.default_rng(9)
    words = rng.integers(0, 2 ** 30, size=37, dtype=np.int64)
    s = np.asarray([0.125], np.float16)
    z = np.asarray([3.0], np.float16)
    out = OPS[kind](words_t(words, cuda_device), torch.from_numpy(s).to(cuda_device),
                    torch.from_numpy(z).to(cuda_device))
    assert_bits(out, oracle.dequantize(kind, words, s, z))
    out0 = OPS[kind](words_t(words, cuda_device), torch.from_numpy(s).to(cuda_device), None)
    assert_bits(out0, oracle.dequantize(kind, words, s, np.zeros(1, np.float16)))


def test_empty_and_misaligned_views(cuda_device):
    e = t4_kernels.dequantize_s4(torch.empty(0, dtype=torch.int32, device=cuda_device),
                                 torch.empty(0, dtype=torch.float16, device=cuda_device),
                                 torch.empty(0, dtype=torch.float16, device=cuda_device))
    assert e.numel() == 0
    rng = np.random.default_rng(11)
    words, s, z = _random_inputs(rng, 1031, "int")
    W = words_t(words, cuda_device)
    S = torch.from_numpy(s).to(cuda_device)
    Z = torch.from_numpy(z).to(cuda_device)
    # views at odd offsets take the scalar path
    out = t4_kernels.dequantize_u4(W[1:], S[1:], Z[1:])
    assert_bits(out, oracle.dequantize("u4", words[1:], s[1:], z[1:]))
    out = t4_kernels.dequantize_s3(W[3:] & 0x3FFFFFFF, S[3:], Z[3:], mode="magic")
    assert_bits(out, oracle.dequantize("s3", words[3:] & 0x3FFFFFFF, s[3:], z[3:], mode="magic"))


def test_batch_stress_one_million(cuda_device):
    """tests/test_dequant_correctness.py:190-194 largest batch, plus random words."""
    n = 1_000_000
    rng = np.random.default_rng(13)
    words = rng.integers(0, 2 ** 32, size=n, dtype=np.int64)
    s = np.full(n, 0.5, np.float16)
    z = np.full(n, 1.0, np.float16)
    W, S, Z = words_t(words, cuda_device), torch.from_numpy(s).to(cuda_device), torch.from_numpy(z).to(cuda_device)
    for kind in ("u4", "s4"):
        assert_bits(OPS[kind](W, S, Z), oracle.dequantize(kind, words, s, z))


def test_bad_arguments_raise(cuda_device):
    w = torch.zeros(8, dtype=torch.int32, device=cuda_device)
    s = torch.ones(8, dtype=torch.float16, device=cuda_device)
    with pytest.raises(RuntimeError):
        t4_kernels.dequantize_u4(w, s[:3], s)           # scale count neither 1 nor numel
    with pytest.raises(RuntimeError):
        t4_kernels.dequantize_u4(w.float(), s, s)       # wrong dtype
    with pytest.raises(RuntimeError):
        t4_kernels.dequantize_u4(w, s, s, mode="fast")  # unknown mode
