"""Drop-in module name of the reference extension (src/setup.py:8-13 builds
``t4_kernels``): code written against the reference keeps ``import t4_kernels``
and gets the B200 kernels of ``t4_cuda_b200`` (plus the fused FP8-weight GEMM,
which the reference does not have)."""

from t4_cuda_b200.ops import (  # noqa: F401
    dequantize_u4,
    dequantize_s4,
    dequantize_s3,
    dequantize_fp8,
    fused_w4a16_gemm_u4,
    fused_w4a16_gemm_s4,
    fused_h17_gemv_s3,
    fused_w8a16_gemm_fp8,
)
