"""The seven ops of the reference's ``t4_kernels`` extension, on B200.

Same names, argument order, output shapes and error type (RuntimeError, as
TORCH_CHECK raises) as src/bindings.cpp:8-260 of kridaydave/t4-cuda.  Every op
validates its tensors, allocates its output with ``torch.empty`` on the input's
device and enqueues the CUDA kernel of libt4b200.so on the current stream of
that device, asynchronously.  There is no CPU path: CPU tensors are rejected
exactly as the reference rejects them.

Extensions, all backward compatible (trailing keyword arguments):
  * ``dequantize_*(..., mode="contract")``: "contract" = fp16(fp32((q-z)*s)),
    what the reference tests assert; "magic" = the reference GPU kernels'
    fp16-FMA arithmetic, bit for bit.  Scale / zero point may also have 1
    element (broadcast), as the reference's CPU oracle allows.
  * ``fused_w4a16_gemm_*``: scales / zero points of shape (N,), (1, N) or
    grouped (K/g, N); zero_points may be None or empty (zero).
  * ``fused_h17_gemv_s3(..., group_size=100)``: any group size (the reference
    hard-codes 100).
"""

import ctypes

import torch

from . import _lib

__all__ = [
    "dequantize_u4", "dequantize_s4", "dequantize_s3", "dequantize_fp8",
    "fused_w4a16_gemm_u4", "fused_w4a16_gemm_s4", "fused_w4a16_gemm_grouped", "fused_h17_gemv_s3",
    "fused_w8a16_gemm_fp8",
    "set_gemv_kernel", "device_error",
]

_GEMV_KERNELS = {"auto": 0, "generic": 1, "stream": 2, "tc_single": 3}


def set_gemv_kernel(which="auto"):
    """Choose the W4A16 matmul kernel process-wide: "auto" (the best kernel that
    applies: for M <= 16 the resident-activation decode kernel, then the
    TMA-streamed split-tile kernel; for M > 16 the tcgen05 GEMM, on CTA pairs
    when M > 128; else generic), "tc_single" (as "auto" but M > 16 always on
    single-CTA tcgen05 tiles), "stream" (the split-tile kernel where it applies)
    or "generic" (the register-streaming kernel).  Returns the previous choice."""
    _check(which in _GEMV_KERNELS, f"which must be one of {sorted(_GEMV_KERNELS)}")
    prev = _lib.load().t4b_set_gemv_kernel(_GEMV_KERNELS[which])
    return {v: k for k, v in _GEMV_KERNELS.items()}[prev]


_INT3_KERNELS = {"stream": 0, "ring": 1, "gemv": 2, "tc": 3}


def set_int3_kernel(which="stream"):
    """Choose the INT3 kernel process-wide: "stream" (the register-streaming
    GEMV, the default) or "ring" (the warp-specialized TMA-ring GEMV where it
    applies, else register streaming) -- under both, M > 16 runs on the tcgen05
    INT3 GEMM where it takes the shape (an even group_size >= 64, N % 8 == 0,
    16-byte aligned operands) -- or "gemv" (register streaming at every M), or
    "tc" (the tcgen05 GEMM at every M where it takes the shape).  Returns the
    previous choice."""
    _check(which in _INT3_KERNELS, f"which must be one of {sorted(_INT3_KERNELS)}")
    prev = _lib.load().t4b_set_int3_kernel(_INT3_KERNELS[which])
    return {v: k for k, v in _INT3_KERNELS.items()}[prev]


def device_error(device=None, clear=True):
    """Device error word of this library's workspace for the current stream of
    ``device`` (0 = no kernel gave up a bounded wait).  Synchronizes the stream."""
    import ctypes
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    out = ctypes.c_uint(0)
    with _on_device(dev):
        st = _lib.load().t4b_device_error(_stream_ptr(dev), ctypes.byref(out), 1 if clear else 0)
    _lib.check(st, "t4b_device_error")
    return out.value


def _check(cond, msg):
    if not cond:
        raise RuntimeError(msg)


def _stream_ptr(device):
    return torch.cuda.current_stream(device).cuda_stream


class _on_device:
    """Make ``device`` current for the launch (like at::cuda::CUDAGuard)."""

    __slots__ = ("idx", "prev")

    def __init__(self, device):
        self.idx = device.index if device.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.idx:
            self.prev = cur
            torch.cuda.set_device(self.idx)

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)


def _mode(mode):
    _check(mode in _lib.MODES, f"mode must be one of {sorted(_lib.MODES)}, got {mode!r}")
    return _lib.MODES[mode]


def _aligned16(t):
    """Contiguous tensor whose data pointer is 16-byte aligned (copy if not)."""
    if not t.is_contiguous():
        t = t.contiguous()
    if t.data_ptr() % 16:
        t = t.clone()
    return t


# --------------------------------------------------------------- dequantize
def _dequant(name, per_word_out, packed_weights, scales, zero_points, mode):
    _check(packed_weights.is_cuda, "packed_weights must be a CUDA tensor")
    _check(scales.is_cuda, "scales must be a CUDA tensor")
    has_zp = zero_points is not None
    if has_zp:
        _check(zero_points.is_cuda, "zero_points must be a CUDA tensor")
    _check(packed_weights.dtype == torch.int32, "packed_weights must be Int32")
    _check(scales.dtype == torch.float16, "scales must be FP16")
    if has_zp:
        _check(zero_points.dtype == torch.float16, "zero_points must be FP16")
    dev = packed_weights.device
    _check(scales.device == dev and (not has_zp or zero_points.device == dev),
           "all tensors must be on the same device")
    n = packed_weights.numel()
    _check(scales.numel() in (1, n), f"scales must have 1 or {n} elements (one per packed word), got {scales.numel()}")
    nz = zero_points.numel() if has_zp else 0
    _check(nz in (0, 1, n), f"zero_points must have 1 or {n} elements (one per packed word), got {nz}")
    out = torch.empty(n * per_word_out, dtype=torch.float16, device=dev)
    if n == 0:
        return out
    w = packed_weights.contiguous()
    s = scales.contiguous()
    z = zero_points.contiguous() if nz else None
    m = _mode(mode)
    lib = _lib.load()
    with _on_device(dev):
        st = getattr(lib, name)(w.data_ptr(), s.data_ptr(), z.data_ptr() if z is not None else None,
                                out.data_ptr(), n, s.numel(), nz, m, _stream_ptr(dev))
    _lib.check(st, name)
    return out


def dequantize_u4(packed_weights, scales, zero_points, mode="contract"):
    """Unsigned INT4 dequantization; out[8i + j] = (nibble j of word i - z_i) * s_i.
    Mirrors bindings.cpp:8-33 (dequantize_lop3_u4_cuda)."""
    return _dequant("t4b_dequantize_u4", 8, packed_weights, scales, zero_points, mode)


def dequantize_s4(packed_weights, scales, zero_points, mode="contract"):
    """Signed (two's complement) INT4 dequantization.  Mirrors bindings.cpp:35-60."""
    return _dequant("t4b_dequantize_s4", 8, packed_weights, scales, zero_points, mode)


def dequantize_s3(packed_weights, scales, zero_points, mode="contract"):
    """Signed INT3 dequantization, 10 values per word (bits 3i..3i+2).
    Mirrors bindings.cpp:134-159."""
    return _dequant("t4b_dequantize_s3", 10, packed_weights, scales, zero_points, mode)


def dequantize_fp8(packed_weights, scales, mode="contract"):
    """FP8-E4M3 (4 bytes per word) dequantization.  Mirrors bindings.cpp:161-183."""
    _check(packed_weights.is_cuda, "packed_weights must be a CUDA tensor")
    _check(scales.is_cuda, "scales must be a CUDA tensor")
    _check(packed_weights.dtype == torch.int32, "packed_weights must be Int32")
    _check(scales.dtype == torch.float16, "scales must be FP16")
    dev = packed_weights.device
    _check(scales.device == dev, "all tensors must be on the same device")
    n = packed_weights.numel()
    _check(scales.numel() in (1, n), f"scales must have 1 or {n} elements (one per packed word), got {scales.numel()}")
    out = torch.empty(n * 4, dtype=torch.float16, device=dev)
    if n == 0:
        return out
    w = packed_weights.contiguous()
    s = scales.contiguous()
    m = _mode(mode)
    with _on_device(dev):
        st = _lib.load().t4b_dequantize_fp8(w.data_ptr(), s.data_ptr(), out.data_ptr(), n, s.numel(), m,
                                            _stream_ptr(dev))
    _lib.check(st, "t4b_dequantize_fp8")
    return out


# --------------------------------------------------------------- fused GEMM
def _group_rows(t, N, K, what):
    """(N,) / (1, N) / (G, N) -> number of rows G, with checks."""
    d = t.dim()
    if d == 1:
        if t.numel() != N:
            _fail(f"{what} of shape (N,) must have N={N} elements, got {t.numel()}")
        return 1
    if d != 2:
        _fail(f"{what} must be 1-D (N,) or 2-D (K/group, N)")
    if t.size(1) != N:
        _fail(f"{what} must have N={N} columns, got {t.size(1)}")
    G = t.size(0)
    if G < 1 or K % G:
        _fail(f"{what}: {G} groups must divide K={K}")
    if (K // G) % 8:
        _fail(f"{what}: group size K/{G}={K // G} must be a multiple of 8")
    return G


_FN = {}      # C entry points by name (ctypes function objects, looked up once)


def _entry(name):
    fn = _FN.get(name)
    if fn is None:
        fn = _FN[name] = getattr(_lib.load(), name)
    return fn


def _fail(msg):
    raise RuntimeError(msg)


def _check_a(A):
    if not A.is_cuda:
        _fail("A must be a CUDA tensor")


def _check_w(A, W_packed, scales, zero_points):
    """The checks of bindings.cpp:64-132 after A's device check, in the same
    order, with messages formatted only on failure; returns (M, N, K, G,
    has_zp)."""
    if not W_packed.is_cuda:
        _fail("W_packed must be a CUDA tensor")
    if not scales.is_cuda:
        _fail("scales must be a CUDA tensor")
    has_zp = zero_points is not None and zero_points.numel() > 0
    if has_zp:
        if not zero_points.is_cuda:
            _fail("zero_points must be a CUDA tensor")
        if zero_points.dtype != torch.float16:
            _fail("zero_points must be FP16")
    if A.dtype != torch.float16:
        _fail("A must be FP16")
    if W_packed.dtype != torch.int32:
        _fail("W_packed must be Int32")
    if scales.dtype != torch.float16:
        _fail("scales must be FP16")
    if A.dim() != 2:
        _fail("A must be a 2-D (M, K) tensor")
    if W_packed.dim() != 2:
        _fail("W_packed must be a 2-D (K/8, N) tensor")
    dev = A.device
    if W_packed.device != dev or scales.device != dev or (has_zp and zero_points.device != dev):
        _fail("all tensors must be on the same device")
    M, K = A.shape
    N = W_packed.size(1)
    if M <= 0 or N <= 0 or K <= 0:
        _fail("Dimensions M, N, K must be positive")
    if K % 8:
        _fail("K must be a multiple of 8 (8 INT4 values per int32 word)")
    if W_packed.size(0) != K // 8:
        _fail(f"W_packed must have K/8={K // 8} rows, got {W_packed.size(0)}")
    G = _group_rows(scales, N, K, "scales")
    if has_zp and _group_rows(zero_points, N, K, "zero_points") != G:
        _fail("zero_points must have the same shape as scales")
    return M, N, K, G, has_zp


def _contig(t):
    return t if t.is_contiguous() else t.contiguous()


def _fused(name, A, W_packed, scales, zero_points):
    # The decode path calls this once per projection per token, so the host
    # work is kept short.
    _check_a(A)
    M, N, K, G, has_zp = _check_w(A, W_packed, scales, zero_points)
    A_ = _aligned16(A)
    W_ = _contig(W_packed)
    S_ = _contig(scales)
    Z_ = _contig(zero_points) if has_zp else None
    dev = A.device
    C = torch.empty((M, N), dtype=torch.float16, device=dev)
    cur = torch.cuda.current_device()
    idx = dev.index if dev.index is not None else cur
    if cur != idx:
        torch.cuda.set_device(idx)
    try:
        st = _entry(name)(A_.data_ptr(), W_.data_ptr(), S_.data_ptr(), Z_.data_ptr() if Z_ is not None else None,
                          C.data_ptr(), M, N, K, K // G, torch._C._cuda_getCurrentRawStream(idx))
    finally:
        if cur != idx:
            torch.cuda.set_device(cur)
    if st:
        _lib.check(st, name)
    return C


def _fused_grouped(A, W_list, scales_list, zero_points_list, signed):
    n = len(W_list)
    if n < 1 or n > GROUPED_MAX:
        _fail(f"a grouped call takes 1 to {GROUPED_MAX} projections, got {n}")
    if len(scales_list) != n or (zero_points_list is not None and len(zero_points_list) != n):
        _fail("W_packed, scales and zero_points lists must have the same length")
    _check_a(A)
    shapes, zs = [], []
    for j in range(n):
        z = zero_points_list[j] if zero_points_list is not None else None
        M, N, K, G, has_zp = _check_w(A, W_list[j], scales_list[j], z)
        shapes.append((N, G))
        zs.append(z if has_zp else None)
    if len({G for _, G in shapes}) != 1:
        _fail("every projection of a grouped call must have the same group size")
    has_zp = zs[0] is not None
    if any((z is not None) != has_zp for z in zs):
        _fail("zero_points must be given for every projection of a grouped call or for none")
    G = shapes[0][1]
    A_ = _aligned16(A)
    Ws = [_contig(w) for w in W_list]
    Ss = [_contig(t) for t in scales_list]
    Zs = [_contig(z) for z in zs] if has_zp else None
    dev = A.device
    Cs = [torch.empty((M, N), dtype=torch.float16, device=dev) for N, _ in shapes]
    vp = ctypes.c_void_p * n
    cur = torch.cuda.current_device()
    idx = dev.index if dev.index is not None else cur
    if cur != idx:
        torch.cuda.set_device(idx)
    try:
        st = _entry("t4b_fused_w4a16_gemm_grouped")(
            A_.data_ptr(), n, vp(*[w.data_ptr() for w in Ws]), vp(*[t.data_ptr() for t in Ss]),
            vp(*[z.data_ptr() for z in Zs]) if Zs is not None else None, vp(*[c.data_ptr() for c in Cs]),
            (ctypes.c_int * n)(*[N for N, _ in shapes]), M, K, K // G, 1 if signed else 0,
            torch._C._cuda_getCurrentRawStream(idx))
    finally:
        if cur != idx:
            torch.cuda.set_device(cur)
    if st:
        _lib.check(st, "t4b_fused_w4a16_gemm_grouped")
    return Cs


_BIND = False      # the torch binding module once looked up (None: not built)


def _binding():
    """The torch binding of the fused W4A16 ops (bind/torch_ops.cpp, built in-tree
    as ``_torch_ops`` next to the library), initialised with the loaded
    library's entry points; None if it has not been built.  It does the same
    checks as ``_fused`` in C++, which takes the per-call host cost of a decode
    step's ~224 calls from ~11 to a few microseconds."""
    global _BIND
    if _BIND is False:
        import ctypes
        import importlib.util
        b = None
        if importlib.util.find_spec(__package__ + "._torch_ops") is not None:
            from . import _torch_ops as b   # a build that does not load is an error, not a fallback
            lib = _lib.load()
            addr = lambda f: ctypes.cast(f, ctypes.c_void_p).value    # noqa: E731
            b.init(addr(lib.t4b_fused_w4a16_gemm_u4), addr(lib.t4b_fused_w4a16_gemm_s4),
                   addr(lib.t4b_fused_w4a16_gemv_allgather), addr(lib.t4b_fused_w4a16_gemm_grouped),
                   addr(lib.t4b_fused_w4a16_gemv_allgather_grouped),
                   addr(lib.t4b_status_string),
                   addr(lib.t4b_last_cuda_error), _lib.T4BError)
        _BIND = b
    return _BIND


def fused_w4a16_gemm_u4(A, W_packed, scales, zero_points):
    """C = A @ dequant_u4(W_packed).  Mirrors bindings.cpp:64-97."""
    b = _BIND if _BIND is not False else _binding()
    if b is not None:
        return b.fused_w4a16_gemm_u4(A, W_packed, scales, zero_points)
    return _fused("t4b_fused_w4a16_gemm_u4", A, W_packed, scales, zero_points)


def fused_w4a16_gemm_s4(A, W_packed, scales, zero_points):
    """C = A @ dequant_s4(W_packed).  Mirrors bindings.cpp:99-132."""
    b = _BIND if _BIND is not False else _binding()
    if b is not None:
        return b.fused_w4a16_gemm_s4(A, W_packed, scales, zero_points)
    return _fused("t4b_fused_w4a16_gemm_s4", A, W_packed, scales, zero_points)


GROUPED_MAX = 4      # T4B_GROUPED_MAX


def grouped_plan(N_list, M, K, group_size, has_zero_points=False):
    """CTAs per projection of the one decode launch that
    ``fused_w4a16_gemm_grouped`` makes for these shapes on the current
    device, or None when it makes one launch per projection instead."""
    n = len(N_list)
    ctas = (ctypes.c_int * max(n, 1))()
    st = _lib.load().t4b_fused_w4a16_gemm_grouped_plan(n, (ctypes.c_int * max(n, 1))(*N_list), M, K, group_size,
                                                        1 if has_zero_points else 0, ctas)
    if st == 4:         # T4B_ERR_UNSUPPORTED
        return None
    _lib.check(st, "t4b_fused_w4a16_gemm_grouped_plan")
    return list(ctas[:n])


def fused_w4a16_gemm_grouped(A, W_list, scales_list, zero_points_list=None, signed=True):
    """Projections that read the same activation, in one call:
    ``[A @ dequant(W) for W in W_list]`` (s4 weights if ``signed``, else u4),
    each with its scales and zero points (``zero_points_list`` None, or one
    tensor per projection; all given or all None/empty), the same K and group
    size.  No counterpart in the reference, whose op takes one projection (a
    layer's q/k/v or gate/up are separate ``fused_w4a16_gemm_{s4,u4}`` calls);
    the results match those calls within the ops' tolerance.  For M <= 16 the
    projections run as one decode launch whose CTAs are shared out by column
    tiles; otherwise as one launch per projection.  Each projection is
    checked as ``fused_w4a16_gemm_{s4,u4}`` checks it."""
    b = _BIND if _BIND is not False else _binding()
    if b is not None:
        return b.fused_w4a16_gemm_grouped(A, list(W_list), list(scales_list),
                                          None if zero_points_list is None else list(zero_points_list),
                                          bool(signed))
    return _fused_grouped(A, W_list, scales_list, zero_points_list, signed)


# ------------------------------------------------------- FP8-E4M3 weight GEMM
def fused_w8a16_gemm_fp8(A, W_packed, scales):
    """C = A @ (E4M3(W_packed) * scales), fp16 in, fp32 accumulate, fp16 out.

    No counterpart op in the reference (it has only the flat dequantize_fp8,
    lop3_dequant.h:93-123): this is the fused path for its E4M3 weight format.
    W_packed int32 [K/4, N]: byte j of word (kw, n) is the E4M3 code of K row
    4 kw + j (the byte order of dequantize_fp8).  scales fp16 (N,), (1, N) or
    (K/g, N).  The weight is fp16(e4m3 * s) with exact E4M3 decoding (subnormal
    codes are values; 0x7F / 0xFF are NaN and propagate) -- unlike the
    reference's CPU dequant, which flushes subnormal codes to 0 and reads the
    NaN codes as 480 (tests/test_dequant_correctness.py:63-84).  The tcgen05
    kernel takes K % 64 == 0, group % 64 == 0 and N % 8 == 0."""
    if not (A.is_cuda and W_packed.is_cuda and scales.is_cuda):
        _fail("A, W_packed and scales must be CUDA tensors")
    if A.dtype != torch.float16:
        _fail("A must be FP16")
    if W_packed.dtype != torch.int32:
        _fail("W_packed must be Int32")
    if scales.dtype != torch.float16:
        _fail("scales must be FP16")
    if A.dim() != 2 or W_packed.dim() != 2:
        _fail("A must be (M, K) and W_packed (K/4, N)")
    dev = A.device
    if W_packed.device != dev or scales.device != dev:
        _fail("all tensors must be on the same device")
    M, K = A.shape
    N = W_packed.size(1)
    if M <= 0 or N <= 0 or K <= 0:
        _fail("Dimensions M, N, K must be positive")
    if K % 4:
        _fail("K must be a multiple of 4 (4 E4M3 values per int32 word)")
    if W_packed.size(0) != K // 4:
        _fail(f"W_packed must have K/4={K // 4} rows, got {W_packed.size(0)}")
    if scales.dim() == 1:
        G = 1
        if scales.numel() != N:
            _fail(f"scales of shape (N,) must have N={N} elements, got {scales.numel()}")
    else:
        if scales.dim() != 2 or scales.size(1) != N or scales.size(0) < 1 or K % scales.size(0):
            _fail("scales must be (N,), (1, N) or (K/group, N)")
        G = scales.size(0)
    A_ = _aligned16(A)
    W_ = W_packed if W_packed.is_contiguous() else W_packed.contiguous()
    S_ = scales if scales.is_contiguous() else scales.contiguous()
    C = torch.empty((M, N), dtype=torch.float16, device=dev)
    cur = torch.cuda.current_device()
    idx = dev.index if dev.index is not None else cur
    if cur != idx:
        torch.cuda.set_device(idx)
    try:
        st = _entry("t4b_fused_w8a16_gemm_fp8")(A_.data_ptr(), W_.data_ptr(), S_.data_ptr(), C.data_ptr(), M, N, K,
                                                K // G, torch._C._cuda_getCurrentRawStream(idx))
    finally:
        if cur != idx:
            torch.cuda.set_device(cur)
    if st:
        _lib.check(st, "fused_w8a16_gemm_fp8")
    return C


# --------------------------------------------------------------- H17 INT3 GEMV
def fused_h17_gemv_s3(A, W_packed, scales, zero_points, group_size=100):
    """C = A @ dequant_s3(W_packed) with per-group scales / zero points.
    Mirrors bindings.cpp:185-250 check for check; ``group_size`` generalises
    the reference's fixed group of 100 (h17_mega_kernel.cu:22)."""
    _check(A.is_cuda, "A must be a CUDA tensor")
    _check(W_packed.is_cuda, "W_packed must be a CUDA tensor")
    _check(scales.is_cuda, "scales must be a CUDA tensor")
    has_zp = zero_points is not None and zero_points.numel() > 0
    if has_zp:
        _check(zero_points.is_cuda, "zero_points must be a CUDA tensor")
        _check(zero_points.dtype == torch.float16, "zero_points must be FP16")
        _check(zero_points.is_contiguous(), "zero_points must be contiguous")
    _check(A.is_contiguous(), "A must be contiguous")
    _check(W_packed.is_contiguous(), "W_packed must be contiguous")
    _check(scales.is_contiguous(), "scales must be contiguous")
    _check(A.dtype == torch.float16, "A must be FP16")
    _check(W_packed.dtype == torch.int32, "W_packed must be Int32")
    _check(scales.dtype == torch.float16, "scales must be FP16")
    _check(A.dim() in (1, 2), "A must be 1D or 2D tensor")
    _check(W_packed.dim() == 2, "W_packed must be a 2D tensor")
    dev = A.device
    _check(W_packed.device == dev and scales.device == dev and (not has_zp or zero_points.device == dev),
           "all tensors must be on the same device")
    M = 1 if A.dim() == 1 else A.size(0)
    K = A.size(0) if A.dim() == 1 else A.size(1)
    N = W_packed.size(1)
    _check(M > 0 and N > 0 and K > 0, "Dimensions M, N, K must be positive")
    _check(K % 10 == 0, "K must be a multiple of 10 for H17 int3 packing")
    _check(W_packed.size(0) == K // 10, "W_packed first dim must equal K/10 (canonical H17 layout)")
    _check(isinstance(group_size, int) and group_size >= 10,
           "group_size must be an int >= 10 (a 10-value word may straddle at most one group boundary)")
    num_groups = (K + group_size - 1) // group_size
    _check(scales.numel() == num_groups * N,
           f"scales must have num_groups * N elements (num_groups = ceil(K/{group_size}))")
    if has_zp:
        _check(zero_points.numel() == num_groups * N, "zero_points must have num_groups * N elements")
    A_ = _aligned16(A)
    C = torch.empty((M, N), dtype=torch.float16, device=dev)
    with _on_device(dev):
        st = _lib.load().t4b_fused_h17_gemv_s3(A_.data_ptr(), W_packed.data_ptr(), scales.data_ptr(),
                                               zero_points.data_ptr() if has_zp else None, C.data_ptr(),
                                               M, N, K, group_size, _stream_ptr(dev))
    _lib.check(st, "t4b_fused_h17_gemv_s3")
    return C
