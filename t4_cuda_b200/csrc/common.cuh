// Shared device helpers and host plumbing for the sm_100a W4A16 / INT3 kernels.
//
// Arithmetic that must be bit-exact is written with explicit-rounding PTX
// (".rn" forms) so the optimizer cannot contract or reorder it.
#pragma once

#include <atomic>

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "t4b200.h"

namespace t4b {

// ---------------------------------------------------------------- host side
// Records a CUDA error for t4b_last_cuda_error() and returns T4B_ERR_CUDA.
int record_cuda_error(cudaError_t err);

// Checks the launch that was just enqueued.
inline int check_launch() {
    cudaError_t err = cudaGetLastError();
    return err == cudaSuccess ? T4B_OK : record_cuda_error(err);
}

// Streaming-multiprocessor count of the current device (cached per device).
int sm_count();

// Per-device record of the dynamic shared memory a kernel has been allowed
// (cudaFuncAttributeMaxDynamicSharedMemorySize applies to the device that is
// current when it is set, so each device needs its own call).
struct SmemLimit {
    int bytes[64] = {0};
};
// Raises `kernel`'s dynamic shared-memory limit on the current device to at
// least `bytes` (a no-op once it is there); thread-safe.  T4B_OK or the
// recorded CUDA error.
int ensure_dynamic_smem(const void* kernel, int bytes, SmemLimit* limit);

// TMA-streamed, SM-balanced W4A16 GEMV (gemv_w4_stream.cu).  Returns
// T4B_ERR_UNSUPPORTED when the shape / alignment does not suit it.
int gemv_w4_stream(bool is_signed, const void* A, const void* W, const void* S, const void* Z, void* C, int M, int N,
                   int K, int group, cudaStream_t stream);

// Decode GEMV with resident activations (M <= 16; M * K <= 32768, or larger
// when the activations still fit in shared memory and N / 16 >= SMs); returns
// T4B_ERR_UNSUPPORTED (without launching) for shapes it does not take.
int gemv_w4_decode(bool is_signed, const void* A, const void* W, const void* S, const void* Z, void* C, int M, int N,
                   int K, int group, cudaStream_t stream);
// T4B_OK when the decode kernel takes the shape (nothing is launched).
int gemv_w4_decode_supported(int M, int N, int K, int group, bool has_zero_points);
// Same kernel with the fused all-gather of T4BGather (epoch-tagged column
// pairs into every rank's receive buffer); T4B_ERR_UNSUPPORTED where the
// decode kernel does not apply.
int gemv_w4_decode_gather(bool is_signed, const void* A, const void* W, const void* S, const void* Z, int M, int N,
                          int K, int group, const T4BGather* g, cudaStream_t stream);
// One decode launch for np projections that read the same A (W, S, C, N:
// np entries each; Z NULL or np entries); T4B_ERR_UNSUPPORTED (nothing
// launched) where the decode kernel does not take the shapes.
int gemv_w4_decode_grouped(bool is_signed, const void* A, int np, const void* const* W, const void* const* S,
                           const void* const* Z, void* const* C, const int* N, int M, int K, int group,
                           cudaStream_t stream);
// The CTAs of each projection of that launch (nothing is launched).
int gemv_w4_decode_grouped_plan(int np, const int* N, int M, int K, int group, bool has_zero_points, int* ctas);
// The same launch with the fused all-gather: projection j's columns go to
// [col_offsets[j], col_offsets[j] + N[j]) of the group buffer of g.
int gemv_w4_decode_gather_grouped(bool is_signed, const void* A, int np, const void* const* W, const void* const* S,
                                  const void* const* Z, const int* N, const int* col_offsets, int M, int K, int group,
                                  const T4BGather* g, cudaStream_t stream);

// Reads (and optionally clears) the decode GEMV's device error word on the
// current device; synchronizes `stream`.
int decode_device_error(cudaStream_t stream, unsigned* out, bool clear);
// Same for the allocation-free GEMV's word (in its fixed scratch array).
int static_scratch_error(cudaStream_t stream, unsigned* out, bool clear);
// Same for the TMA-ring INT3 GEMV's word.
int int3_device_error(cudaStream_t stream, unsigned* out, bool clear);

// Prefill GEMM on tcgen05 / TMEM (M > 16, K % 64 == 0, group % 64 == 0);
// T4B_ERR_UNSUPPORTED (without launching) for shapes it does not take.
// allow_pairs: M > 128 runs on CTA pairs (cta_group::2); else single CTAs.
int gemm_w4_tc(bool is_signed, const void* A, const void* W, const void* S, const void* Z, void* C, int M, int N, int K,
               int group, bool allow_pairs, cudaStream_t stream);
int gemm_tc_device_error(cudaStream_t stream, unsigned* out, bool clear);

// INT3 (H17 packing) prefill GEMM on tcgen05 / TMEM (M > 16, K % 10 == 0, an
// even group >= 64, N % 8 == 0, 16-byte aligned operands);
// T4B_ERR_UNSUPPORTED (without launching) for shapes it does not take.
// any_m: also M <= 16 (else T4B_ERR_UNSUPPORTED for those).
int gemm_int3_tc(const void* A, const void* W, const void* S, const void* Z, void* C, int M, int N, int K, int group,
                 bool any_m, cudaStream_t stream);
int int3_tc_device_error(cudaStream_t stream, unsigned* out, bool clear);

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// Clusters of `ks` CTAs (1 x 1 x ks) of `kernel` (dynamic shared memory
// `smem`, `threads` a CTA) that can be resident at once on the current device
// (cudaOccupancyMaxActiveClusters; 0 if none or on error), cached per device
// and size in `cache`.  ks: 2..8.
struct ClusterCapacityCache {
    std::atomic<int> n[64][9];
    SmemLimit limit;            // the kernel's dynamic shared-memory attribute, per device
};
int max_active_clusters(const void* kernel, int smem, int threads, int ks, ClusterCapacityCache* cache);

// Division by a runtime constant d >= 1 for numerators n < 2^31:
// n / d == (umulhi(n, mul) + n) >> shift  (Granlund & Montgomery, PLDI 1994).
struct FastDiv {
    uint32_t d, mul, shift;
};
inline FastDiv make_fastdiv(uint32_t d) {
    uint32_t l = 0;
    while ((1ull << l) < d) ++l;
    const uint64_t m = ((1ull << 32) * ((1ull << l) - d)) / d + 1;
    return FastDiv{d, (uint32_t)m, l};
}
__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv& f) {
    return (__umulhi(n, f.mul) + n) >> f.shift;
}

// -------------------------------------------------------------- device side
// lop3.b32 with a compile-time truth table.
template <int LUT>
__device__ __forceinline__ uint32_t lop3(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, %4;" : "=r"(d) : "r"(a), "r"(b), "r"(c), "n"(LUT));
    return d;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// Packed fp16 arithmetic with round-to-nearest-even, never fused.
__device__ __forceinline__ uint32_t h2_sub(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t h2_mul(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t h2_fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ uint32_t h2_dup(uint16_t bits) { return (uint32_t)bits * 0x10001u; }
__device__ __forceinline__ uint32_t h2_pack(uint16_t lo, uint16_t hi) { return (uint32_t)lo | ((uint32_t)hi << 16); }
__device__ __forceinline__ uint16_t h_bits(__half h) { return __half_as_ushort(h); }
__device__ __forceinline__ float h_to_f(uint16_t bits) { return __half2float(__ushort_as_half(bits)); }

// Two fp32 values -> packed fp16 pair, each rounded to nearest even.
__device__ __forceinline__ uint32_t f2_to_h2(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}

// fp16 constants (bit patterns, duplicated into both halves).
constexpr uint32_t H2_1024 = 0x64006400u;   // 1024.0
constexpr uint32_t H2_1028 = 0x64046404u;   // 1028.0
constexpr uint32_t H2_1032 = 0x64086408u;   // 1032.0

// ---------------------------------------------------------------------------
// Exact integer extraction of 4-bit weights into fp16 pairs.
//
// Word w holds eight nibbles n0..n7 (n_j at bits 4j..4j+3).  The results are
// four fp16x2 registers holding the integer weights EXACTLY:
//     p[0] = (q0, q4), p[1] = (q1, q5), p[2] = (q2, q6), p[3] = (q3, q7)
// with q = n (unsigned) or the two's-complement value of n (signed).
//
// Method: OR a nibble into the mantissa of 1024.0 (exponent 0x64) so the fp16
// value is 1024 + n (low nibble) or 1024 + 16 n (nibble shifted up by 4), then
// subtract / rescale exactly.  For signed weights the nibble's top bit is
// flipped on the way in (n ^ 8 = q + 8), so the same subtraction yields q.
// Only one shift per word is needed.
template <bool SIGNED>
__device__ __forceinline__ void unpack_w4_exact(uint32_t w, uint32_t (&p)[4]) {
    // truth table 0xEA = (a & b) | c ; 0x6A = (a ^ c) & b | (c & ~b)
    constexpr uint32_t LO_MASK = 0x000F000Fu, HI_MASK = 0x00F000F0u;
    const uint32_t w8 = w >> 8;
    uint32_t lo0, hi0, lo1, hi1;
    if (SIGNED) {
        lo0 = lop3<0x6A>(w, LO_MASK, 0x64086408u);    // 1024 + (n ^ 8)
        hi0 = lop3<0x6A>(w, HI_MASK, 0x64806480u);    // 1024 + 16 (n ^ 8)
        lo1 = lop3<0x6A>(w8, LO_MASK, 0x64086408u);
        hi1 = lop3<0x6A>(w8, HI_MASK, 0x64806480u);
        // (1024 + (q+8)) - 1032 = q ;  (1024 + 16(q+8)) / 16 - 72 = q
        p[0] = h2_sub(lo0, H2_1032);
        p[1] = h2_fma(hi0, 0x2C002C00u /*1/16*/, 0xD480D480u /*-72*/);
        p[2] = h2_sub(lo1, H2_1032);
        p[3] = h2_fma(hi1, 0x2C002C00u, 0xD480D480u);
    } else {
        lo0 = lop3<0xEA>(w, LO_MASK, H2_1024);        // 1024 + n
        hi0 = lop3<0xEA>(w, HI_MASK, H2_1024);        // 1024 + 16 n
        lo1 = lop3<0xEA>(w8, LO_MASK, H2_1024);
        hi1 = lop3<0xEA>(w8, HI_MASK, H2_1024);
        p[0] = h2_sub(lo0, H2_1024);
        p[1] = h2_fma(hi0, 0x2C002C00u, 0xD400D400u /*-64*/);
        p[2] = h2_sub(lo1, H2_1024);
        p[3] = h2_fma(hi1, 0x2C002C00u, 0xD400D400u);
    }
}

// The reference GPU arithmetic ("magic" mode): raw = B + q built in fp16 by a
// LOP3 against a magic exponent, then ONE fp16 FMA raw * s + bias where
// bias = fp16(fp32(-B - z) * s) (B = 1024 unsigned, 1032 signed).  Pairs as
// in unpack_w4_exact.  Restates src/kernels/lop3_dequant.h:10-53 and
// lop3_dequant.cu:23-32.
template <bool SIGNED>
__device__ __forceinline__ void dequant_w4_magic(uint32_t w, uint32_t s2, uint32_t bias2, uint32_t (&p)[4]) {
    constexpr uint32_t MASK = 0x000F000Fu;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t x = w >> (4 * j);
        const uint32_t raw = SIGNED ? lop3<0x6A>(x, MASK, H2_1032) : lop3<0xEA>(x, MASK, H2_1024);
        p[j] = h2_fma(raw, s2, bias2);
    }
}

// Signed 3-bit fields: word w holds e_0..e_9 (e_i at bits 3i..3i+2).  Returns
// five fp16x2 registers holding the integers exactly:
//     p[i] = (q_i, q_{i+5}),  i = 0..4.
// The word is first re-spread so elements 5..9 start at bit 16 (x = bits
// 0..14 of w in the low half, bits 15..29 in the high half); fields 0..2 of
// each half are then ORed straight into the mantissa of 1024 (value 1024 +
// 2^(3i) (e ^ 4)), fields 3..4 after one shift.
__device__ __forceinline__ void unpack_s3_exact(uint32_t w, uint32_t (&p)[5]) {
    const uint32_t x = ((w << 1) & 0x7FFF0000u) | (w & 0x00007FFFu);
    const uint32_t x9 = x >> 9;
    // field i at bit offset 3i of each half: raw = 1024 + 2^(3i) * (e ^ 4)
    const uint32_t r0 = lop3<0x6A>(x, 0x00070007u, 0x64046404u);   // 1024 + (e^4)
    const uint32_t r1 = lop3<0x6A>(x, 0x00380038u, 0x64206420u);   // 1024 + 8 (e^4)
    const uint32_t r2 = lop3<0x6A>(x, 0x01C001C0u, 0x65006500u);   // 1024 + 64 (e^4)
    const uint32_t r3 = lop3<0x6A>(x9, 0x00070007u, 0x64046404u);
    const uint32_t r4 = lop3<0x6A>(x9, 0x00380038u, 0x64206420u);
    // q = (raw - 1024) / 2^(3i) - 4 = raw * 2^-3i - (1024 * 2^-3i + 4)
    p[0] = h2_sub(r0, H2_1028);
    p[1] = h2_fma(r1, 0x30003000u /*1/8*/, 0xD820D820u /*-(128+4)*/);
    p[2] = h2_fma(r2, 0x24002400u /*1/64*/, 0xCD00CD00u /*-(16+4)*/);
    p[3] = h2_sub(r3, H2_1028);
    p[4] = h2_fma(r4, 0x30003000u, 0xD820D820u);
}

// Reference GPU arithmetic for s3 (lop3_dequant.h:55-85, lop3_dequant.cu:99-108):
// raw = 1028 + q via LOP3 0x6A against 0x6404, one fp16 FMA with
// bias = fp16(fp32(-1028 - z) * s).  Pairs as in unpack_s3_exact.
__device__ __forceinline__ void dequant_s3_magic(uint32_t w, uint32_t s2, uint32_t bias2, uint32_t (&p)[5]) {
#pragma unroll
    for (int i = 0; i < 5; ++i) {
        const uint32_t pair = ((w >> (3 * i)) & 0x7u) | (((w >> (3 * i + 15)) & 0x7u) << 16);
        const uint32_t raw = lop3<0x6A>(pair, 0x00070007u, 0x64046404u);
        p[i] = h2_fma(raw, s2, bias2);
    }
}

}  // namespace t4b
