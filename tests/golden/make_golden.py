#!/usr/bin/env python3
"""Generate the golden vectors under tests/golden/ from the reference's OWN
CPU functions (kridaydave/t4-cuda), imported from a read-only checkout.

Run in a container that has the reference checkout, passing its location
(or setting T4B_REFERENCE):

    python tests/golden/make_golden.py <reference checkout>

The outputs are committed; the tests read only the outputs, never the
reference.  Every case records which reference function produced it.

Reference functions used (paths inside the reference project):
  * tests/test_dequant_correctness.py:18-38   cpu_dequantize (u4)
  * tests/test_dequant_correctness.py:40-61   cpu_dequantize_s3 (non-negative words only:
                                              its uint32 wrap at :58 breaks negatives)
  * tests/test_dequant_correctness.py:63-84   cpu_dequantize_fp8
  * harness/verify_dequant.py:20-44           unpack_uint32_to_{u4,s4}, dequantize_{u4,s4}_reference
  * tests/test_fused_gemm_correctness.py:11-36 dequantize_ref / cpu_reference_gemm
  * harness/verify_fused_gemm.py:4-50         dequantize_{u4,s4}_ref (seed-42 1024x1024 case)
  * tests/test_h17_fused_int3_gemv.py:426-472 pack / quantize_int3_canonical / cpu_ref_h17_gemv
"""

import hashlib
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "tests"))
    sys.path.insert(0, os.path.join(ref_root, "harness"))
    # test_dequant_correctness.py exits at import time without its extension or
    # a GPU; give it an empty stand-in module and a CUDA probe that says yes.
    # Only its pure-CPU functions are called below.
    sys.modules.setdefault("t4_kernels", types.ModuleType("t4_kernels"))
    real_probe = torch.cuda.is_available
    torch.cuda.is_available = lambda: True
    try:
        import test_dequant_correctness as tdc
    finally:
        torch.cuda.is_available = real_probe
    import test_fused_gemm_correctness as tfg
    import test_h17_fused_int3_gemv as th17
    import verify_dequant as vd
    import verify_fused_gemm as vfg
    return tdc, tfg, th17, vd, vfg


def u32(x):
    return int(x) & 0xFFFFFFFF


def i32_tensor(words):
    """Pack uint32 values into an int32 tensor through int64 (keeps bit 31)."""
    return torch.tensor([u32(w) for w in words], dtype=torch.int64).to(torch.int32)


def f16_bits(t):
    return np.asarray(t, dtype=np.float16).view(np.uint16).reshape(-1).tolist()


def sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(np.asarray(a)).tobytes())
    return h.hexdigest()


def dequant_cases(tdc, vd):
    cases = []

    def add(name, words, scales, zeros, kind, expected16, source):
        cases.append({
            "name": name, "kind": kind,
            "words": [u32(w) for w in words],
            "scales_f16": f16_bits(np.asarray(scales, np.float16)),
            "zeros_f16": f16_bits(np.asarray(zeros, np.float16)),
            "expected_f16": f16_bits(expected16),
            "source": source,
        })

    def ref_u4(words, s, z):
        p = i32_tensor(words)
        st = torch.tensor(np.asarray(s, np.float16))
        zt = torch.tensor(np.asarray(z, np.float16))
        return tdc.cpu_dequantize(p, st, zt, is_signed=False).numpy().reshape(-1)

    def ref_s4(words, s, z):
        # harness/verify_dequant.py evaluates (s4 - z) * s in Python floats; the
        # product is exact, then rounded to fp32 and fp16 like the test oracle.
        s = np.broadcast_to(np.asarray(s, np.float16), (len(words),))
        z = np.broadcast_to(np.asarray(z, np.float16), (len(words),))
        vals = vd.dequantize_s4_reference([u32(w) for w in words],
                                          [float(x) for x in s], [float(x) for x in z])
        return np.asarray(vals, np.float64).astype(np.float32).astype(np.float16)

    src_u4 = "tests/test_dequant_correctness.py:18-38 cpu_dequantize(is_signed=False)"
    src_s4 = "harness/verify_dequant.py:36-44 dequantize_s4_reference"

    # tests/test_dequant_correctness.py:139-163 known-answer words
    kats = [("KAT H4", 0xA7C13E59, 0.25, 2.0), ("all zeros", 0x00000000, 1.0, 0.0),
            ("all ones", 0xFFFFFFFF, 1.0, 0.0), ("identity", 0x76543210, 1.0, 0.0)]
    for name, w, s, z in kats:
        add(name + " u4", [w], [s], [z], "u4", ref_u4([w], [s], [z]), src_u4)
        add(name + " s4", [w], [s], [z], "s4", ref_s4([w], [s], [z]), src_s4)

    # :165-180 exhaustive nibble sweep
    sweep = [sum(n << (4 * i) for i in range(8)) for n in range(16)]
    ones, zs = [1.0] * 16, [0.0] * 16
    add("nibble sweep u4", sweep, ones, zs, "u4", ref_u4(sweep, ones, zs), src_u4)
    add("nibble sweep s4", sweep, ones, zs, "s4", ref_s4(sweep, ones, zs), src_s4)

    # :190-194 batch stress (identity word, s=0.5, z=1), small batches
    for b in (1, 256):
        w = [0x76543210] * b
        s, z = [0.5] * b, [1.0] * b
        add(f"batch {b} u4", w, s, z, "u4", ref_u4(w, s, z), src_u4)
        add(f"batch {b} s4", w, s, z, "s4", ref_s4(w, s, z), src_s4)

    # :196-210 scale edges (u4): 0, 65000 (overflows to inf), 1e-5 (fp16 subnormal)
    for s in (0.0, 65000.0, 1e-5):
        add(f"scale edge {s:g} u4", [0x76543210], [s], [0.0], "u4",
            ref_u4([0x76543210], [s], [0.0]), src_u4)

    # harness/verify_dequant.py:86-119 asymmetric KATs (printed answers in
    # results/t4_colab_runtime_logs/02_verify_dequant.log:50-59)
    add("harness KAT u4 0xA7C13E59", [0xA7C13E59], [0.25], [2.0], "u4",
        np.asarray(vd.dequantize_u4_reference([0xA7C13E59], [0.25], [2.0]), np.float64)
        .astype(np.float32).astype(np.float16), "harness/verify_dequant.py:28-33")
    add("harness KAT s4 0xF817E29A", [0xF817E29A], [0.5], [0.0], "s4",
        ref_s4([0xF817E29A], [0.5], [0.0]), src_s4)

    # harness/verify_lop3_standalone.py:38-40 and :67-69 four-word KATs (inputs
    # restated: that script needs a GPU at import), answers by verify_dequant.py
    w = [0xA7C13E59, 0x12345678, 0xFEDCBA98, 0x0F0F0F0F]
    s, z = [0.25, 0.5, 0.1, 1.0], [2.0, 0.0, 1.0, 0.0]
    sf = [float(np.float16(x)) for x in s]
    exp = np.asarray(vd.dequantize_u4_reference(w, sf, z), np.float64).astype(np.float32).astype(np.float16)
    add("lop3 standalone u4", w, s, z, "u4", exp, "harness/verify_dequant.py:28-33")
    w = [0xF817E29A, 0x87654321, 0x98BADCFE, 0xF0F0F0F0]
    s, z = [0.5, 0.25, 0.2, 0.5], [0.0, 1.0, -1.0, 0.0]
    add("lop3 standalone s4", w, s, z, "s4", ref_s4(w, s, z), src_s4)
    return cases


def fuzz_arrays(tdc):
    """:182-188 random fuzz: full-range words, scale and zero point randn*5."""
    g = torch.Generator().manual_seed(0)
    n = 10000
    words = torch.randint(-2147483648, 2147483647, (n,), dtype=torch.int32, generator=g)
    s = (torch.randn(n, generator=g) * 5.0).half()
    z = (torch.randn(n, generator=g) * 5.0).half()
    exp_u4 = tdc.cpu_dequantize(words, s, z, is_signed=False).numpy().reshape(-1)
    return words.numpy(), s.numpy(), z.numpy(), exp_u4


def s3_cases(tdc):
    """cpu_dequantize_s3 on words whose ten fields are all 0..3 (its uint32
    wrap only bites negative fields); ordering and scaling are pinned here,
    negatives by the H17 GEMV cases."""
    rng = np.random.default_rng(3)
    fields = rng.integers(0, 4, size=(64, 10))
    words = (fields << (3 * np.arange(10))[None, :]).sum(axis=1)
    s = rng.standard_normal(64).astype(np.float16)
    z = rng.integers(-2, 3, size=64).astype(np.float16)
    exp = tdc.cpu_dequantize_s3(i32_tensor(words), torch.tensor(s), torch.tensor(z)).numpy().reshape(-1)
    return {"name": "s3 non-negative fields", "kind": "s3", "words": [u32(w) for w in words],
            "scales_f16": f16_bits(s), "zeros_f16": f16_bits(z), "expected_f16": f16_bits(exp),
            "source": "tests/test_dequant_correctness.py:40-61 cpu_dequantize_s3"}


def fp8_case(tdc):
    words = [b | (b + 1) << 8 | (b + 2) << 16 | (b + 3) << 24 for b in range(0, 256, 4)]
    cyc = [1.0, 0.5, -2.0, 0.001, 3.0]
    s = np.asarray([cyc[i % len(cyc)] for i in range(len(words))], np.float16)
    with np.errstate(over="ignore", invalid="ignore"):
        exp = tdc.cpu_dequantize_fp8(i32_tensor(words), torch.tensor(s)).numpy().reshape(-1)
    # That oracle computes 2.0**(exp - 7) on a uint32 exponent (:81), which
    # wraps for exponent fields 1..6 and yields inf; only bytes whose exponent
    # field is 0 or >= 7 carry a usable answer.
    e = (np.arange(256) >> 3) & 0xF
    valid = [bool(x == 0 or x >= 7) for x in e]
    return {"name": "fp8 all 256 bytes", "kind": "fp8", "words": words,
            "scales_f16": f16_bits(s), "zeros_f16": [], "expected_f16": f16_bits(exp),
            "valid": valid,
            "source": "tests/test_dequant_correctness.py:63-84 cpu_dequantize_fp8"}


def gemm_cases(tfg):
    out = {}

    def case(tag, M, K, N, signed, seed, full_range, zp=True, A=None):
        g = torch.Generator().manual_seed(seed)
        if A is None:
            A = torch.randn(M, K, generator=g).half()
        if full_range:
            W = torch.randint(0, 2 ** 32, (K // 8, N), dtype=torch.int64, generator=g).to(torch.int32)
        else:   # the reference's own generator never sets bit 31 (:43)
            W = torch.randint(0, 2 ** 31 - 1, (K // 8, N), dtype=torch.int32, generator=g)
        s = (torch.randn(1, N, generator=g) * 0.1).half()
        z = torch.randint(0, 16, (1, N), generator=g).half() if zp else torch.zeros(1, N).half()
        c16 = tfg.cpu_reference_gemm(A, W, s, z, signed=signed)
        c32 = torch.matmul(A.float(), tfg.dequantize_ref(W, s, z, signed=signed).float())
        out[tag + "_A"] = A.numpy()
        out[tag + "_W"] = W.numpy()
        out[tag + "_s"] = s.numpy()
        out[tag + "_z"] = z.numpy()
        out[tag + "_c16"] = c16.numpy()
        out[tag + "_c32"] = c32.numpy()
        out[tag + "_signed"] = np.asarray(int(signed))

    case("small_u4", 1, 8, 4, False, 1, False)          # :88 "Known Small Matrix"
    case("edge_u4", 1, 8, 1, False, 2, False)           # :113 "Minimum K, Single N"
    case("batch_s4", 4, 256, 64, True, 3, True)         # :90-91 shape family, full range
    case("nozp_s4", 8, 128, 32, True, 4, True, zp=False)
    case("identity_u4", 8, 8, 8, False, 5, False, A=torch.eye(8).half())   # :68-84
    return out


def harness_seed42_case(vfg):
    """harness/verify_fused_gemm.py:58-91 recipe on the CPU generator (the
    reference drew it on a GPU): seed 42, M=1, K=N=1024.  Inputs are
    regenerated by the test; their hash guards generator drift."""
    torch.manual_seed(42)
    M, K, N = 1, 1024, 1024
    A = torch.randn((M, K), dtype=torch.float16)
    W = torch.randint(0, 0x7FFFFFFF, (K // 8, N), dtype=torch.int32)
    scale = torch.rand((N,), dtype=torch.float16) * 0.1 + 0.05
    zero = torch.randint(0, 8, (N,), dtype=torch.float16)
    res = {"input_sha256": sha(A.numpy(), W.numpy(), scale.numpy(), zero.numpy())}
    for signed, fn in ((False, vfg.dequantize_u4_ref), (True, vfg.dequantize_s4_ref)):
        Wd = fn(W, scale, zero, K, N)
        res["u4s4"[2 * signed:2 * signed + 2] + "_c16"] = f16_bits(torch.matmul(A.float(), Wd.float()).half())
        res["u4s4"[2 * signed:2 * signed + 2] + "_c32"] = torch.matmul(A.float(), Wd.float()).numpy().reshape(-1).tolist()
    return res


def int3_cases(th17):
    out = {}

    def case(tag, seed, M, K, N, group, scale_a=0.5, zp=True):
        rng = np.random.default_rng(seed)
        A = (rng.standard_normal((M, K)) * scale_a).astype(np.float32)
        W = (rng.standard_normal((N, K)) * 0.5).astype(np.float32)
        packed, s_gn, z_gn = th17.quantize_int3_canonical(W, group_size=group)
        if not zp:
            z_gn = np.zeros_like(z_gn)
        c = th17.cpu_ref_h17_gemv(A, packed, s_gn, z_gn, group_size=group)
        out[tag + "_A"] = A
        out[tag + "_W"] = packed.astype(np.uint32).view(np.int32)
        out[tag + "_s"] = s_gn.astype(np.float32)
        out[tag + "_z"] = z_gn.astype(np.float32)
        out[tag + "_c"] = c.astype(np.float32)
        out[tag + "_group"] = np.asarray(group)

    case("gate", 20260731, 1, 200, 64, 100)      # :492-527, the reference GPU gate
    case("g128", 7, 2, 260, 16, 128)             # group 128: words straddle groups
    case("nozp", 11, 3, 100, 8, 100, zp=False)
    return out


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("T4B_REFERENCE")
    if not ref_root:
        raise SystemExit("usage: make_golden.py <reference checkout> (or set T4B_REFERENCE)")
    tdc, tfg, th17, vd, vfg = _import_reference(ref_root)

    cases = dequant_cases(tdc, vd)
    cases.append(s3_cases(tdc))
    cases.append(fp8_case(tdc))
    with open(os.path.join(HERE, "dequant_kats.json"), "w") as f:
        json.dump({"generator": "tests/golden/make_golden.py", "cases": cases}, f)

    words, s, z, exp = fuzz_arrays(tdc)
    np.savez_compressed(os.path.join(HERE, "dequant_fuzz_u4.npz"), words=words, scales=s,
                        zeros=z, expected=exp)

    np.savez_compressed(os.path.join(HERE, "gemm_cases.npz"), **gemm_cases(tfg))
    with open(os.path.join(HERE, "gemm_seed42.json"), "w") as f:
        json.dump(harness_seed42_case(vfg), f)
    np.savez_compressed(os.path.join(HERE, "int3_cases.npz"), **int3_cases(th17))
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
