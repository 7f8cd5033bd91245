"""ctypes binding of the C ABI in include/t4b200.h (libt4b200.so, built in-tree).

There is no fallback: if the library is missing the first op call raises.
"""

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libt4b200.so")

MODES = {"contract": 0, "magic": 1}

_vp, _i32, _i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64

# name -> argument types (restype is int for all compute entry points)
SIGNATURES = {
    "t4b_dequantize_u4": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _vp],
    "t4b_dequantize_s4": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _vp],
    "t4b_dequantize_s3": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _vp],
    "t4b_dequantize_fp8": [_vp, _vp, _vp, _i64, _i64, _i32, _vp],
    "t4b_fused_w4a16_gemm_u4": [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp],
    "t4b_fused_w4a16_gemm_s4": [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp],
    "t4b_fused_w4a16_gemm_grouped": [_vp, _i32, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp],
    "t4b_fused_w4a16_gemm_grouped_plan": [_i32, _vp, _i32, _i32, _i32, _i32, _vp],
    "t4b_fused_h17_gemv_s3": [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp],
    "t4b_fused_w8a16_gemm_fp8": [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp],
    "t4b_fused_w4a16_gemv_noalloc": [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _vp],
    "t4b_fused_w4a16_gemv_allgather": [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _vp, _vp],
    "t4b_fused_w4a16_gemv_allgather_supported": [_i32, _i32, _i32, _i32, _i32],
    "t4b_fused_w4a16_gemv_allgather_grouped": [_vp, _i32, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp,
                                               _vp],
    "t4b_ipc_alloc": [ctypes.c_size_t, ctypes.POINTER(_vp)],
    "t4b_ipc_free": [_vp],
    "t4b_ipc_handle": [_vp, _vp],
    "t4b_ipc_open": [_vp, ctypes.POINTER(_vp)],
    "t4b_ipc_close": [_vp],
}


class T4BGather(ctypes.Structure):
    """include/t4b200.h T4BGather: receive buffers, output and counter of a fused all-gather."""
    _fields_ = [
        ("recv", _vp * 8),
        ("out", _vp),
        ("counter", _vp),
        ("world", ctypes.c_int),
        ("rank", ctypes.c_int),
        ("n_total", ctypes.c_int),
        ("col_offset", ctypes.c_int),
        ("barrier", ctypes.c_int),
    ]

_lock = threading.Lock()
_lib = None


class T4BError(RuntimeError):
    """A non-zero status from the C ABI (a RuntimeError, like TORCH_CHECK)."""


def load():
    """Load libt4b200.so once and declare every entry point's signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is not built; run `python -m t4_cuda_b200.build` (needs nvcc). "
                "There is no CPU fallback for these ops.")
        lib = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        lib.t4b_status_string.argtypes = [ctypes.c_int]
        lib.t4b_status_string.restype = ctypes.c_char_p
        lib.t4b_last_cuda_error.argtypes = []
        lib.t4b_last_cuda_error.restype = ctypes.c_int
        lib.t4b_version.argtypes = []
        lib.t4b_version.restype = ctypes.c_int
        lib.t4b_set_gemv_kernel.argtypes = [ctypes.c_int]
        lib.t4b_set_gemv_kernel.restype = ctypes.c_int
        lib.t4b_set_int3_kernel.argtypes = [ctypes.c_int]
        lib.t4b_set_int3_kernel.restype = ctypes.c_int
        lib.t4b_device_error.argtypes = [_vp, ctypes.POINTER(ctypes.c_uint), ctypes.c_int]
        lib.t4b_device_error.restype = ctypes.c_int
        lib.t4b_workspace_bytes.argtypes = [_vp, ctypes.POINTER(ctypes.c_size_t)]
        lib.t4b_workspace_bytes.restype = ctypes.c_int
        _lib = lib
    return _lib


def check(status, op):
    if status != 0:
        lib = load()
        msg = lib.t4b_status_string(status).decode()
        cuda = lib.t4b_last_cuda_error() if status == 5 else 0
        raise T4BError(f"{op}: {msg} (status {status}" + (f", cudaError {cuda})" if cuda else ")"))
