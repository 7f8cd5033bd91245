"""B200-native (sm_100a) W4A16 / INT3 quantized matmul -- a drop-in for the
``t4_kernels`` extension of kridaydave/t4-cuda.

    import t4_cuda_b200 as t4k            # or: import t4_kernels (repo-root shim)
    C = t4k.fused_w4a16_gemm_s4(A, W_packed, scales, zero_points)

The CUDA kernels live in ``libt4b200.so`` (C ABI: include/t4b200.h), built
in-tree by ``python -m t4_cuda_b200.build``.  ``t4_cuda_b200.shard`` adds the
column-sharded multi-GPU wrapper.
"""

from .ops import (  # noqa: F401
    dequantize_u4,
    dequantize_s4,
    dequantize_s3,
    dequantize_fp8,
    fused_w4a16_gemm_u4,
    fused_w4a16_gemm_s4,
    fused_w4a16_gemm_grouped,
    fused_h17_gemv_s3,
    fused_w8a16_gemm_fp8,
    set_gemv_kernel,
    set_int3_kernel,
    device_error,
)
from ._lib import LIB_PATH, T4BError, load as load_library  # noqa: F401

__version__ = "1.0.0"
