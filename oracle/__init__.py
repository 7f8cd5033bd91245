"""CPU oracle for the W4A16 / INT3 hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the arithmetic of the reference project
(kridaydave/t4-cuda) for the packed-weight dequantization ops, the fused
W4A16 GEMV/GEMM and the H17 INT3 GEMV.  Every function cites the reference
file:line it follows.

Who may use it: only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``
(its ``cpu_baseline`` leg and its ``--impl reference`` arm).  It is the checker,
never the thing measured on the GPU and never a fallback: the product package
``t4_cuda_b200`` does not import it.

Parity is pinned: ``tests/test_oracle_golden.py`` checks these functions
against golden vectors produced by the reference's own CPU functions
(``tests/golden/make_golden.py``), and the GPU tests additionally check the
"magic" mode against the reference's CUDA kernels compiled from source by
``oracle/build_ref.sh`` into ``oracle/_ref/``.
"""

from .dequant import (  # noqa: F401
    MAGIC_BIAS,
    as_u32,
    unpack_u4,
    unpack_s4,
    unpack_s3,
    dequantize,
    dequantize_fp8,
    fp16_bits,
)
from .gemm import (  # noqa: F401
    pack_int4,
    expand_scales,
    dequant_w4_matrix,
    ref_w4_gemm,
)
from .int3 import (  # noqa: F401
    pack_int3,
    quantize_int3,
    unpack_int3_matrix,
    dequant_int3_matrix,
    ref_int3_gemv,
)
from .fp8 import (  # noqa: F401
    e4m3_to_float,
    pack_fp8,
    unpack_fp8_codes,
    dequant_fp8_matrix,
    ref_fp8_gemm,
)
