// C-ABI shim over the reference project's own CUDA launchers -- TEST
// INFRASTRUCTURE ONLY (a GPU-side checker, never shipped or measured).
//
// oracle/build_ref.sh compiles this file together with the reference's
// unmodified kernel sources (src/kernels/lop3_dequant.cu,
// src/kernels/fused_w4a16_gemm.cu, src/kernels/h17_mega_kernel.cu, taken
// from where they lie in the reference checkout) into oracle/_ref/libt4ref.so.
// The launchers it forwards to are declared in src/kernels/lop3_dequant.h:126-136,
// src/kernels/fused_w4a16_gemm.h:24-46 and src/kernels/h17_mega_kernel.h:22-30;
// their arguments are plain device pointers, so the shim only casts.
//
// Input contracts the caller must honour (the reference kernels do not check):
//   dequant: scales / zero points hold one fp16 per packed word;
//   fused W4A16: N % 4 == 0 (the kernel returns early per column before a
//     full-warp shuffle), per-column scales and zero points of length N;
//   H17: K % 10 == 0, scales (and zero points, or null) of ceil(K/100) x N.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "fused_w4a16_gemm.h"
#include "h17_mega_kernel.h"
#include "lop3_dequant.h"

extern "C" {

int t4ref_dequant(int kind, const void* packed, void* out, const void* scale, const void* zero, int num_words,
                  void* stream) {
    auto p = static_cast<const uint32_t*>(packed);
    auto o = static_cast<half*>(out);
    auto s = static_cast<const half*>(scale);
    auto z = static_cast<const half*>(zero);
    auto st = static_cast<cudaStream_t>(stream);
    switch (kind) {
        case 0: launch_lop3_dequant_u4(p, o, s, z, num_words, st); break;
        case 1: launch_lop3_dequant_s4(p, o, s, z, num_words, st); break;
        case 2: launch_lop3_dequant_s3(p, o, s, z, num_words, st); break;
        case 3: launch_lop3_dequant_fp8(p, o, s, num_words, st); break;
        default: return -1;
    }
    return (int)cudaGetLastError();
}

int t4ref_fused_w4a16(int is_signed, const void* A, const void* W, const void* scale, const void* zero, void* C, int M,
                      int N, int K, void* stream) {
    auto a = static_cast<const half*>(A);
    auto w = static_cast<const uint32_t*>(W);
    auto s = static_cast<const half*>(scale);
    auto z = static_cast<const half*>(zero);
    auto c = static_cast<half*>(C);
    auto st = static_cast<cudaStream_t>(stream);
    if (is_signed)
        launch_fused_w4a16_gemm_s4(a, w, s, z, c, M, N, K, st);
    else
        launch_fused_w4a16_gemm_u4(a, w, s, z, c, M, N, K, st);
    return (int)cudaGetLastError();
}

int t4ref_h17_gemv(const void* A, const void* W, const void* scale, const void* zero, void* C, int M, int N, int K,
                   int num_groups, void* stream) {
    launch_h17_gemv_s3(static_cast<const half*>(A), static_cast<const uint32_t*>(W), static_cast<const half*>(scale),
                       static_cast<const half*>(zero), static_cast<half*>(C), M, N, K, num_groups,
                       static_cast<cudaStream_t>(stream));
    return (int)cudaGetLastError();
}

}  // extern "C"
