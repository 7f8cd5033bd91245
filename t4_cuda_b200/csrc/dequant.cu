// Flat dequantization of packed u4 / s4 / s3 / fp8-e4m3 words to fp16.
//
// Replaces the reference's one-thread-per-word kernels
// (src/kernels/lop3_dequant.cu:9-148) with an HBM-streaming design: each
// thread handles 4 consecutive words per iteration -- one 128-bit load of
// words, 64-bit loads of the per-word scales / zero points and 128-bit
// streaming stores of the 32..80 output bytes -- in a grid-stride loop sized
// to the SM count.  Traffic per word: 4 B in + 2 B scale + 2 B zero point +
// 16 B (u4/s4), 20 B (s3) or 8 B (fp8) out.
//
// Two arithmetic modes (T4B_MODE_*):
//   contract  fp16_rn(fp32_rn((q - z) * s)), bit-exact with the reference's
//             CPU oracle (tests/test_dequant_correctness.py:18-84);
//   magic     the reference GPU kernels' own arithmetic, bit-exact with them.
#include "common.cuh"

namespace t4b {
namespace {

enum Fmt { U4 = 0, S4 = 1, S3 = 2, FP8 = 3 };

template <int F> struct Fmt_;
template <> struct Fmt_<U4>  { static constexpr int kElems = 8,  kRegs = 4; static constexpr float kBias = 1024.f; };
template <> struct Fmt_<S4>  { static constexpr int kElems = 8,  kRegs = 4; static constexpr float kBias = 1032.f; };
template <> struct Fmt_<S3>  { static constexpr int kElems = 10, kRegs = 5; static constexpr float kBias = 1028.f; };
template <> struct Fmt_<FP8> { static constexpr int kElems = 4,  kRegs = 2; static constexpr float kBias = 0.f; };

// fp32 product of the contract rule for one exact integer q.
// When z is a multiple of 2^-8, q - z is exact in fp32 (|q - z| < 2^16) and two
// fp32 roundings-free steps give fp32_rn((q - z) * s).  Otherwise the product
// is formed exactly in fp64 (at most 39 significant bits) and rounded once.
__device__ __forceinline__ float contract_f32(float q, float s, float z, bool z_fast) {
    if (z_fast) return __fmul_rn(__fsub_rn(q, z), s);
    return __double2float_rn(((double)q - (double)z) * (double)s);
}

// Contract-mode pair: exact integer pair (fp16x2) -> fp16x2 result.
__device__ __forceinline__ uint32_t contract_pair(uint32_t qpair, float s, float z, bool z_fast) {
    const float2 q = __half22float2(*reinterpret_cast<const __half2*>(&qpair));
    return f2_to_h2(contract_f32(q.x, s, z, z_fast), contract_f32(q.y, s, z, z_fast));
}

// One word -> Fmt_<F>::kRegs packed fp16 pairs in natural element order.
template <int F, int MODE>
__device__ __forceinline__ void dequant_word(uint32_t w, uint16_t sb, uint16_t zb, uint32_t (&o)[Fmt_<F>::kRegs]) {
    const float s = h_to_f(sb);
    if constexpr (F == FP8) {
        if constexpr (MODE == T4B_MODE_MAGIC) {
            // lop3_dequant.h:93-123: fp16 pattern ((b & 0x7F) << 7) + 0x2000 | sign << 15,
            // then fma.rn.f16x2(raw, s, +0)
            const uint32_t s2 = h2_dup(sb);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t x = (w >> (16 * h)) & 0xFFFFu;
                const uint32_t em = ((x & 0x7Fu) << 7) | (((x >> 8) & 0x7Fu) << 23);
                const uint32_t sg = ((x & 0x80u) << 8) | (((x >> 8) & 0x80u) << 24);
                o[h] = h2_fma((em + 0x20002000u) | sg, s2, 0u);
            }
        } else {
            // tests/test_dequant_correctness.py:74-82: 0 when the exponent field is 0,
            // else (-1)^sign * 2^(e-7) * (1 + m/8); v * s is exact in fp32.
            float v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t b = (w >> (8 * j)) & 0xFFu;
                const uint32_t e = (b >> 3) & 0xFu;
                const uint32_t bits = ((b >> 7) << 31) | ((e + 120u) << 23) | ((b & 7u) << 20);
                v[j] = e ? __fmul_rn(__uint_as_float(bits), s) : __fmul_rn(0.0f, s);
            }
            o[0] = f2_to_h2(v[0], v[1]);
            o[1] = f2_to_h2(v[2], v[3]);
        }
    } else {
        constexpr bool SIGNED = (F != U4);
        constexpr int NP = (F == S3) ? 5 : 4;
        uint32_t p[NP];
        if constexpr (MODE == T4B_MODE_MAGIC) {
            const float z = h_to_f(zb);
            const float bias = __fmul_rn(__fsub_rn(-Fmt_<F>::kBias, z), s);
            const uint32_t s2 = h2_dup(sb);
            const uint32_t b2 = h2_dup(__half_as_ushort(__float2half_rn(bias)));
            if constexpr (F == S3) dequant_s3_magic(w, s2, b2, p);
            else dequant_w4_magic<SIGNED>(w, s2, b2, p);
        } else {
            if constexpr (F == S3) unpack_s3_exact(w, p);
            else unpack_w4_exact<SIGNED>(w, p);
            const float z = h_to_f(zb);
            if (z == rintf(z) && fabsf(z) <= 2032.f) {
                // q - z is an exact small integer in fp16 and (q - z) * s has at
                // most 22 significant bits: one fp16 rounding == the contract.
                const uint32_t s2 = h2_dup(sb), z2 = h2_dup(zb);
#pragma unroll
                for (int i = 0; i < NP; ++i) p[i] = h2_mul(h2_sub(p[i], z2), s2);
            } else {
                const float t = z * 256.f;
                const bool z_fast = (t == rintf(t));
#pragma unroll
                for (int i = 0; i < NP; ++i) p[i] = contract_pair(p[i], s, z, z_fast);
            }
        }
        // pairs (q_i, q_{i+NP}) -> natural order
        if constexpr (F == S3) {
            o[0] = prmt(p[0], p[1], 0x5410);
            o[1] = prmt(p[2], p[3], 0x5410);
            o[2] = prmt(p[4], p[0], 0x7610);
            o[3] = prmt(p[1], p[2], 0x7632);
            o[4] = prmt(p[3], p[4], 0x7632);
        } else {
            o[0] = prmt(p[0], p[1], 0x5410);
            o[1] = prmt(p[2], p[3], 0x5410);
            o[2] = prmt(p[0], p[1], 0x7632);
            o[3] = prmt(p[2], p[3], 0x7632);
        }
    }
}

template <int F, int MODE>
__device__ __forceinline__ void scalar_word(const uint32_t* __restrict__ words, const uint16_t* __restrict__ scales,
                                            const uint16_t* __restrict__ zeros, uint16_t* __restrict__ out,
                                            int64_t i, int s_stride, int z_stride) {
    constexpr int R = Fmt_<F>::kRegs;
    const uint16_t sb = scales[i * s_stride];
    const uint16_t zb = zeros ? zeros[i * z_stride] : (uint16_t)0;
    uint32_t o[R];
    dequant_word<F, MODE>(words[i], sb, zb, o);
    uint16_t* dst = out + i * Fmt_<F>::kElems;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        dst[2 * r] = (uint16_t)(o[r] & 0xFFFFu);
        dst[2 * r + 1] = (uint16_t)(o[r] >> 16);
    }
}

template <int F, int MODE, bool VEC>
__global__ void __launch_bounds__(256)
dequant_kernel(const uint32_t* __restrict__ words, const uint16_t* __restrict__ scales,
               const uint16_t* __restrict__ zeros, uint16_t* __restrict__ out,
               int64_t n, int s_stride, int z_stride) {
    constexpr int R = Fmt_<F>::kRegs;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
    int64_t tail_start = 0;
    if constexpr (VEC) {
        const int64_t ngroups = n >> 2;
        tail_start = ngroups << 2;
        const uint16_t s_bcast = s_stride ? (uint16_t)0 : scales[0];
        const uint16_t z_bcast = (zeros && !z_stride) ? zeros[0] : (uint16_t)0;
        for (int64_t g = tid; g < ngroups; g += nthreads) {
            const uint4 wv = __ldcs(reinterpret_cast<const uint4*>(words) + g);
            uint16_t sb[4], zb[4];
            if (s_stride) {
                const uint2 sv = __ldcs(reinterpret_cast<const uint2*>(scales) + g);
                sb[0] = sv.x & 0xFFFF; sb[1] = sv.x >> 16; sb[2] = sv.y & 0xFFFF; sb[3] = sv.y >> 16;
            } else {
                sb[0] = sb[1] = sb[2] = sb[3] = s_bcast;
            }
            if (zeros && z_stride) {
                const uint2 zv = __ldcs(reinterpret_cast<const uint2*>(zeros) + g);
                zb[0] = zv.x & 0xFFFF; zb[1] = zv.x >> 16; zb[2] = zv.y & 0xFFFF; zb[3] = zv.y >> 16;
            } else {
                zb[0] = zb[1] = zb[2] = zb[3] = z_bcast;
            }
            uint32_t o[4 * R];
            const uint32_t wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                uint32_t ok[R];
                dequant_word<F, MODE>(wa[k], sb[k], zb[k], ok);
#pragma unroll
                for (int r = 0; r < R; ++r) o[k * R + r] = ok[r];
            }
            uint4* dst = reinterpret_cast<uint4*>(out + g * 4 * Fmt_<F>::kElems);
#pragma unroll
            for (int v = 0; v < R; ++v) __stcs(dst + v, make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]));
        }
    }
    for (int64_t i = tail_start + tid; i < n; i += nthreads)
        scalar_word<F, MODE>(words, scales, zeros, out, i, s_stride, z_stride);
}

template <int F, int MODE>
int launch_mode(const void* words, const void* scales, const void* zeros, void* out, int64_t n,
                int s_stride, int z_stride, bool vec, cudaStream_t stream) {
    const int threads = 256;
    const int64_t units = vec ? (n >> 2) + (n & 3) : n;
    int64_t blocks = (units + threads - 1) / threads;
    const int64_t cap = (int64_t)sm_count() * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    auto* w = static_cast<const uint32_t*>(words);
    auto* s = static_cast<const uint16_t*>(scales);
    auto* z = static_cast<const uint16_t*>(zeros);
    auto* o = static_cast<uint16_t*>(out);
    if (vec)
        dequant_kernel<F, MODE, true><<<(unsigned)blocks, threads, 0, stream>>>(w, s, z, o, n, s_stride, z_stride);
    else
        dequant_kernel<F, MODE, false><<<(unsigned)blocks, threads, 0, stream>>>(w, s, z, o, n, s_stride, z_stride);
    return check_launch();
}

template <int F>
int dequantize(const void* words, const void* scales, const void* zeros, void* out, int64_t n,
               int64_t n_scales, int64_t n_zeros, int mode, void* stream_) {
    if (n < 0) return T4B_ERR_INVALID_VALUE;
    if (mode != T4B_MODE_CONTRACT && mode != T4B_MODE_MAGIC) return T4B_ERR_INVALID_VALUE;
    if (n == 0) return T4B_OK;
    if (!words || !scales || !out) return T4B_ERR_NULL_POINTER;
    if (n_scales != 1 && n_scales != n) return T4B_ERR_INVALID_VALUE;
    if (n_zeros != 0 && n_zeros != 1 && n_zeros != n) return T4B_ERR_INVALID_VALUE;
    if (n_zeros != 0 && !zeros) return T4B_ERR_NULL_POINTER;
    if (!aligned(words, 4) || !aligned(scales, 2) || !aligned(out, 2) || (zeros && !aligned(zeros, 2)))
        return T4B_ERR_MISALIGNED;
    const void* z = n_zeros ? zeros : nullptr;
    const int s_stride = (n_scales == 1 && n > 1) ? 0 : 1;
    const int z_stride = (n_zeros == 1 && n > 1) ? 0 : 1;
    const bool vec = aligned(words, 16) && aligned(out, 16) && (s_stride == 0 || aligned(scales, 8)) &&
                     (!z || z_stride == 0 || aligned(z, 8));
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    if (mode == T4B_MODE_MAGIC) return launch_mode<F, T4B_MODE_MAGIC>(words, scales, z, out, n, s_stride, z_stride, vec, stream);
    return launch_mode<F, T4B_MODE_CONTRACT>(words, scales, z, out, n, s_stride, z_stride, vec, stream);
}

}  // namespace
}  // namespace t4b

extern "C" {

int t4b_dequantize_u4(const void* words, const void* scales, const void* zero_points, void* out,
                      int64_t num_words, int64_t num_scales, int64_t num_zero_points, int mode, void* stream) {
    return t4b::dequantize<t4b::U4>(words, scales, zero_points, out, num_words, num_scales, num_zero_points, mode, stream);
}

int t4b_dequantize_s4(const void* words, const void* scales, const void* zero_points, void* out,
                      int64_t num_words, int64_t num_scales, int64_t num_zero_points, int mode, void* stream) {
    return t4b::dequantize<t4b::S4>(words, scales, zero_points, out, num_words, num_scales, num_zero_points, mode, stream);
}

int t4b_dequantize_s3(const void* words, const void* scales, const void* zero_points, void* out,
                      int64_t num_words, int64_t num_scales, int64_t num_zero_points, int mode, void* stream) {
    return t4b::dequantize<t4b::S3>(words, scales, zero_points, out, num_words, num_scales, num_zero_points, mode, stream);
}

int t4b_dequantize_fp8(const void* words, const void* scales, void* out, int64_t num_words,
                       int64_t num_scales, int mode, void* stream) {
    return t4b::dequantize<t4b::FP8>(words, scales, nullptr, out, num_words, num_scales, 0, mode, stream);
}

}  // extern "C"
