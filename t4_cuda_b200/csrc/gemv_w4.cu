// Fused W4A16 decode GEMV / skinny GEMM:  C[M, N] = A[M, K] x dequant(W)[K, N].
//
// Replaces src/kernels/fused_w4a16_gemm.cu:15-222 (one 4-byte load per thread,
// 64 threads per column, fp16 products).  This kernel is built for HBM
// streaming on B200:
//
//  * A warp owns a 64-column strip and walks K in steps of 4 packed word rows
//    (32 K).  Lane (r = lane/4, c = lane%4) loads two 128-bit vectors per step:
//    words (kw0 + c, n0 + 4r .. 4r+3) and (kw0 + c, n0 + 32 + 4r .. +3), so a
//    warp reads 4 rows x 256 contiguous bytes.
//  * Each word is turned into 8 EXACT fp16 integers with one shift and four
//    LOP3s against a magic exponent (common.cuh), zero point subtracted and
//    the group scale applied with one fp16 multiply: the weight is
//    fp16_rn((q - z) * s), the dequant contract, held in registers.
//  * Those registers ARE the A fragment of mma.m16n8k16 (weights on the MMA's
//    M side = 16 output columns, batch rows on its N side = 8 rows, fp32
//    accumulation).  The K order inside a fragment is permuted to the
//    nibble-pair order the LOP3 produces; the activation fragment is permuted
//    the same way with two PRMTs, so no shuffles are needed.
//  * K is split across the warps of a CTA and across the CTAs of a thread-block
//    cluster (grid.y = cluster size); partial sums are reduced in shared
//    memory and then across the cluster through distributed shared memory.
//    There is no global workspace and no atomic.
//  * M > 16 runs ceil(M/16) row chunks in grid.z (the tensor-core GEMM is the
//    intended path for prefill shapes).
#include "common.cuh"

#include <atomic>
#include <cooperative_groups.h>

namespace cg = cooperative_groups;

namespace t4b {
namespace {

constexpr int kWarps = 8;          // warps per CTA
constexpr int kTileN = 64;         // output columns per CTA
constexpr int kNB = 4;             // steps of loads kept in flight per lane
constexpr int kStreamMaxM = 16;    // the streaming kernel serves one 16-row chunk

std::atomic<int> g_gemv_kernel{T4B_GEMV_AUTO};

struct GemvParams {
    const uint16_t* A;       // [M, K]
    const uint32_t* W;       // [K/8, N]
    const uint16_t* S;       // [G, N]
    const uint16_t* Z;       // [G, N] or null
    uint16_t* C;             // [M, N]
    int M, N, K, KW;         // KW = K / 8
    FastDiv group_words;     // group_size / 8
    int steps_per_warp;      // steps of 4 word rows per warp
    int total_steps;         // ceil(KW / 4)
};

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ld_stream(const uint32_t* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

// Column of the tile (0..63) held by word slot j (0..7) of lane row r.
__device__ __forceinline__ int slot_col(int r, int j) { return (j < 4) ? 4 * r + j : 32 + 4 * r + (j - 4); }

// Everything one lane needs for one K step.
template <int MT, bool HAS_ZP>
struct StepData {
    uint32_t w[8];           // words, slot j -> column slot_col(r, j)
    uint32_t s[4];           // 8 scales as fp16 pairs (slot 2i, 2i+1)
    uint32_t z[HAS_ZP ? 4 : 1];
    uint4 a[MT];             // 8 activations of row m0 + 8 mt + r at K = 8 (kw0 + c)
};

template <int MT, bool HAS_ZP, bool VEC>
__device__ __forceinline__ void load_step(const GemvParams& p, StepData<MT, HAS_ZP>& d, int step, bool in_range,
                                          int r, int c, int n0, int m0) {
    const int kw = 4 * step + c;
    const bool vk = in_range && kw < p.KW;
    const int g = vk ? (int)fdiv((uint32_t)kw, p.group_words) : 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int col = n0 + 32 * h + 4 * r;
        if (VEC) {
            const bool v = vk && col < p.N;
            const uint4 wv = v ? ld_stream(p.W + (size_t)kw * p.N + col) : make_uint4(0, 0, 0, 0);
            d.w[4 * h + 0] = wv.x; d.w[4 * h + 1] = wv.y; d.w[4 * h + 2] = wv.z; d.w[4 * h + 3] = wv.w;
            const uint2 sv = v ? __ldg(reinterpret_cast<const uint2*>(p.S + (size_t)g * p.N + col)) : make_uint2(0, 0);
            d.s[2 * h] = sv.x; d.s[2 * h + 1] = sv.y;
            if constexpr (HAS_ZP) {
                const uint2 zv = v ? __ldg(reinterpret_cast<const uint2*>(p.Z + (size_t)g * p.N + col)) : make_uint2(0, 0);
                d.z[2 * h] = zv.x; d.z[2 * h + 1] = zv.y;
            }
        } else {
            uint16_t sh[4], zh[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const bool v = vk && (col + j) < p.N;
                d.w[4 * h + j] = v ? __ldg(p.W + (size_t)kw * p.N + col + j) : 0u;
                sh[j] = v ? __ldg(p.S + (size_t)g * p.N + col + j) : (uint16_t)0;
                zh[j] = (HAS_ZP && v) ? __ldg(p.Z + (size_t)g * p.N + col + j) : (uint16_t)0;
            }
            d.s[2 * h] = h2_pack(sh[0], sh[1]); d.s[2 * h + 1] = h2_pack(sh[2], sh[3]);
            if constexpr (HAS_ZP) { d.z[2 * h] = h2_pack(zh[0], zh[1]); d.z[2 * h + 1] = h2_pack(zh[2], zh[3]); }
        }
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
        const int m = m0 + 8 * mt + r;
        d.a[mt] = (vk && m < p.M) ? __ldg(reinterpret_cast<const uint4*>(p.A + (size_t)m * p.K + 8 * kw))
                                  : make_uint4(0, 0, 0, 0);
    }
}

template <int MT, bool SIGNED, bool HAS_ZP>
__device__ __forceinline__ void compute_step(const StepData<MT, HAS_ZP>& d, float (&acc)[MT][4][4]) {
    // Activation fragments: k-half h uses pairs (a[2h], a[2h+4]) and (a[2h+1], a[2h+5]).
    uint32_t b[MT][2][2];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
        b[mt][0][0] = prmt(d.a[mt].x, d.a[mt].z, 0x5410);
        b[mt][0][1] = prmt(d.a[mt].x, d.a[mt].z, 0x7632);
        b[mt][1][0] = prmt(d.a[mt].y, d.a[mt].w, 0x5410);
        b[mt][1][1] = prmt(d.a[mt].y, d.a[mt].w, 0x7632);
    }
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        uint32_t P[2][4];   // scaled weight pairs of slots 2t (row r) and 2t+1 (row r+8)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int j = 2 * t + e;
            const uint32_t spair = d.s[j >> 1];
            const uint32_t s2 = prmt(spair, spair, (j & 1) ? 0x3232 : 0x1010);
            unpack_w4_exact<SIGNED>(d.w[j], P[e]);
            if constexpr (HAS_ZP) {
                const uint32_t zpair = d.z[j >> 1];
                const uint32_t z2 = prmt(zpair, zpair, (j & 1) ? 0x3232 : 0x1010);
#pragma unroll
                for (int i = 0; i < 4; ++i) P[e][i] = h2_sub(P[e][i], z2);
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) P[e][i] = h2_mul(P[e][i], s2);
        }
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
                mma_16816(acc[mt][t], P[0][2 * h], P[1][2 * h], P[0][2 * h + 1], P[1][2 * h + 1], b[mt][h][0], b[mt][h][1]);
    }
}

template <int MT, bool SIGNED, bool HAS_ZP, bool VEC, bool CLUSTER>
__global__ void __launch_bounds__(kWarps * 32)
gemv_w4_kernel(const GemvParams p) {
    constexpr int MR = 8 * MT;                    // batch rows per CTA
    constexpr int RED_STRIDE = MR + 1;            // padded row of the reduction buffer
    __shared__ float red[kWarps][kTileN * RED_STRIDE];

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r = lane >> 2, c = lane & 3;
    const int n0 = blockIdx.x * kTileN;
    const int m0 = blockIdx.z * MR;
    const int u = blockIdx.y * kWarps + warp;
    const int s_begin = u * p.steps_per_warp;
    const int s_end = min(s_begin + p.steps_per_warp, p.total_steps);

    float acc[MT][4][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int t = 0; t < 4; ++t)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[mt][t][i] = 0.f;

    StepData<MT, HAS_ZP> buf[kNB];
#pragma unroll
    for (int i = 0; i < kNB; ++i)
        load_step<MT, HAS_ZP, VEC>(p, buf[i], s_begin + i, s_begin + i < s_end, r, c, n0, m0);
    for (int s = s_begin; s < s_end; s += kNB) {
#pragma unroll
        for (int i = 0; i < kNB; ++i) {
            if (s + i < s_end) {
                compute_step<MT, SIGNED, HAS_ZP>(buf[i], acc);
                const int nxt = s + i + kNB;
                load_step<MT, HAS_ZP, VEC>(p, buf[i], nxt, nxt < s_end, r, c, n0, m0);
            }
        }
    }

    // Warp partials -> shared memory.  d0,d1: (column slot 2t, rows 2c, 2c+1);
    // d2,d3: (column slot 2t+1, rows 2c, 2c+1) of m-tile mt.
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int c0 = slot_col(r, 2 * t), c1 = slot_col(r, 2 * t + 1);
            const int mm = 8 * mt + 2 * c;
            red[warp][c0 * RED_STRIDE + mm] = acc[mt][t][0];
            red[warp][c0 * RED_STRIDE + mm + 1] = acc[mt][t][1];
            red[warp][c1 * RED_STRIDE + mm] = acc[mt][t][2];
            red[warp][c1 * RED_STRIDE + mm + 1] = acc[mt][t][3];
        }
    __syncthreads();
    constexpr int OUTS = kTileN * MR;
    for (int o = threadIdx.x; o < OUTS; o += kWarps * 32) {
        const int idx = (o / MR) * RED_STRIDE + (o % MR);
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) v += red[w][idx];
        red[0][idx] = v;
    }

    if constexpr (CLUSTER) {
        cg::cluster_group cluster = cg::this_cluster();
        cluster.sync();
        const int nranks = (int)cluster.num_blocks();
        const int rank = (int)cluster.block_rank();
        const int per = (OUTS + nranks - 1) / nranks;
        const int o_end = min(OUTS, (rank + 1) * per);
        for (int o = rank * per + threadIdx.x; o < o_end; o += kWarps * 32) {
            const int col = o / MR, mm = o % MR;
            const int idx = col * RED_STRIDE + mm;
            float v = 0.f;
            for (int q = 0; q < nranks; ++q) v += cluster.map_shared_rank(&red[0][0], q)[idx];
            const int m = m0 + mm, n = n0 + col;
            if (m < p.M && n < p.N) p.C[(size_t)m * p.N + n] = __half_as_ushort(__float2half_rn(v));
        }
        cluster.sync();   // keep this CTA's shared memory alive until every rank has read it
    } else {
        __syncthreads();
        for (int o = threadIdx.x; o < OUTS; o += kWarps * 32) {
            const int col = o / MR, mm = o % MR;
            const int m = m0 + mm, n = n0 + col;
            if (m < p.M && n < p.N)
                p.C[(size_t)m * p.N + n] = __half_as_ushort(__float2half_rn(red[0][col * RED_STRIDE + mm]));
        }
    }
}

template <int MT, bool SIGNED, bool HAS_ZP, bool VEC>
int launch_gemv(const GemvParams& p, int splits, cudaStream_t stream) {
    const dim3 block(kWarps * 32);
    const dim3 grid((p.N + kTileN - 1) / kTileN, splits, (p.M + 8 * MT - 1) / (8 * MT));
    if (splits == 1) {
        gemv_w4_kernel<MT, SIGNED, HAS_ZP, VEC, false><<<grid, block, 0, stream>>>(p);
        return check_launch();
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = splits;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t err = cudaLaunchKernelEx(&cfg, gemv_w4_kernel<MT, SIGNED, HAS_ZP, VEC, true>, p);
    if (err != cudaSuccess) return record_cuda_error(err);
    return check_launch();
}

template <int MT, bool SIGNED, bool HAS_ZP>
int dispatch_vec(const GemvParams& p, bool vec, int splits, cudaStream_t s) {
    return vec ? launch_gemv<MT, SIGNED, HAS_ZP, true>(p, splits, s) : launch_gemv<MT, SIGNED, HAS_ZP, false>(p, splits, s);
}

template <bool SIGNED>
int fused_gemm(const void* A, const void* W, const void* S, const void* Z, void* C, int M, int N, int K, int group,
               void* stream_) {
    if (M < 1 || N < 1 || K < 8 || (K % 8) != 0) return T4B_ERR_INVALID_VALUE;
    if (group < 8 || (group % 8) != 0 || (K % group) != 0) return T4B_ERR_INVALID_VALUE;
    if (!A || !W || !S || !C) return T4B_ERR_NULL_POINTER;
    if (!aligned(A, 16) || !aligned(W, 4) || !aligned(S, 2) || !aligned(C, 2) || (Z && !aligned(Z, 2)))
        return T4B_ERR_MISALIGNED;
    const int choice = g_gemv_kernel.load();
    if ((choice == T4B_GEMV_AUTO || choice == T4B_GEMV_TC_SINGLE) && M > kStreamMaxM) {
        const int st = gemm_w4_tc(SIGNED, A, W, S, Z, C, M, N, K, group, choice == T4B_GEMV_AUTO,
                                  static_cast<cudaStream_t>(stream_));
        if (st != T4B_ERR_UNSUPPORTED) return st;
    }
    if ((choice == T4B_GEMV_AUTO || choice == T4B_GEMV_TC_SINGLE) && M <= kStreamMaxM) {
        const int st = gemv_w4_decode(SIGNED, A, W, S, Z, C, M, N, K, group, static_cast<cudaStream_t>(stream_));
        if (st != T4B_ERR_UNSUPPORTED) return st;
    }
    if ((choice == T4B_GEMV_AUTO || choice == T4B_GEMV_TC_SINGLE || choice == T4B_GEMV_STREAM) && M <= kStreamMaxM) {
        const int st = gemv_w4_stream(SIGNED, A, W, S, Z, C, M, N, K, group, static_cast<cudaStream_t>(stream_));
        if (st != T4B_ERR_UNSUPPORTED) return st;
    }
    GemvParams p;
    p.A = static_cast<const uint16_t*>(A);
    p.W = static_cast<const uint32_t*>(W);
    p.S = static_cast<const uint16_t*>(S);
    p.Z = static_cast<const uint16_t*>(Z);
    p.C = static_cast<uint16_t*>(C);
    p.M = M; p.N = N; p.K = K; p.KW = K / 8;
    p.group_words = make_fastdiv((uint32_t)(group / 8));
    p.total_steps = (p.KW + 3) / 4;
    const bool vec = (N % 4 == 0) && aligned(W, 16) && aligned(S, 8) && (!Z || aligned(Z, 8));
    const int mt = (M <= 8) ? 1 : 2;
    const int tiles = (N + kTileN - 1) / kTileN;
    const int chunks = (M + 8 * mt - 1) / (8 * mt);
    // Aim for about two resident CTAs per SM, at most 8 CTAs per cluster and at
    // least one K step per warp.
    int splits = (2 * sm_count() + tiles * chunks - 1) / (tiles * chunks);
    if (splits > 8) splits = 8;
    while (splits > 1 && splits * kWarps > p.total_steps) --splits;
    if (splits < 1) splits = 1;
    const int warps = splits * kWarps;
    p.steps_per_warp = (p.total_steps + warps - 1) / warps;
    cudaStream_t s = static_cast<cudaStream_t>(stream_);
    if (mt == 1) return Z ? dispatch_vec<1, SIGNED, true>(p, vec, splits, s) : dispatch_vec<1, SIGNED, false>(p, vec, splits, s);
    return Z ? dispatch_vec<2, SIGNED, true>(p, vec, splits, s) : dispatch_vec<2, SIGNED, false>(p, vec, splits, s);
}

// Argument checks of one projection of a grouped call, as fused_gemm's.
int check_grouped(const void* A, int n, const void* const* W, const void* const* S, const void* const* Z,
                  void* const* C, const int* N, int M, int K, int group) {
    if (n < 1 || n > T4B_GROUPED_MAX || M < 1 || K < 8 || (K % 8) != 0) return T4B_ERR_INVALID_VALUE;
    if (group < 8 || (group % 8) != 0 || (K % group) != 0) return T4B_ERR_INVALID_VALUE;
    if (!A || !W || !S || !C || !N) return T4B_ERR_NULL_POINTER;
    if (!aligned(A, 16)) return T4B_ERR_MISALIGNED;
    for (int j = 0; j < n; ++j) {
        if (N[j] < 1) return T4B_ERR_INVALID_VALUE;
        if (!W[j] || !S[j] || !C[j] || (Z && !Z[j])) return T4B_ERR_NULL_POINTER;
        if (!aligned(W[j], 4) || !aligned(S[j], 2) || !aligned(C[j], 2) || (Z && !aligned(Z[j], 2)))
            return T4B_ERR_MISALIGNED;
    }
    return T4B_OK;
}

template <bool SIGNED>
int fused_grouped(const void* A, int n, const void* const* W, const void* const* S, const void* const* Z,
                  void* const* C, const int* N, int M, int K, int group, void* stream_) {
    const int st = check_grouped(A, n, W, S, Z, C, N, M, K, group);
    if (st != T4B_OK) return st;
    const int choice = g_gemv_kernel.load();
    if ((choice == T4B_GEMV_AUTO || choice == T4B_GEMV_TC_SINGLE) && M <= kStreamMaxM) {
        const int g = gemv_w4_decode_grouped(SIGNED, A, n, W, S, Z, C, N, M, K, group,
                                             static_cast<cudaStream_t>(stream_));
        if (g != T4B_ERR_UNSUPPORTED) return g;
    }
    for (int j = 0; j < n; ++j) {
        const int s = fused_gemm<SIGNED>(A, W[j], S[j], Z ? Z[j] : nullptr, C[j], M, N[j], K, group, stream_);
        if (s != T4B_OK) return s;
    }
    return T4B_OK;
}

}  // namespace
}  // namespace t4b

extern "C" {

int t4b_fused_w4a16_gemm_grouped(const void* A, int n, const void* const* W_packed, const void* const* scales,
                                 const void* const* zero_points, void* const* C, const int* N, int M, int K,
                                 int group_size, int is_signed, void* stream) {
    return is_signed ? t4b::fused_grouped<true>(A, n, W_packed, scales, zero_points, C, N, M, K, group_size, stream)
                     : t4b::fused_grouped<false>(A, n, W_packed, scales, zero_points, C, N, M, K, group_size, stream);
}

int t4b_fused_w4a16_gemm_grouped_plan(int n, const int* N, int M, int K, int group_size, int has_zero_points,
                                      int* ctas) {
    if (n < 1 || n > T4B_GROUPED_MAX || M < 1 || K < 8 || (K % 8) != 0) return T4B_ERR_INVALID_VALUE;
    if (group_size < 8 || (group_size % 8) != 0 || (K % group_size) != 0) return T4B_ERR_INVALID_VALUE;
    if (!N || !ctas) return T4B_ERR_NULL_POINTER;
    for (int j = 0; j < n; ++j)
        if (N[j] < 1) return T4B_ERR_INVALID_VALUE;
    if (M > t4b::kStreamMaxM) return T4B_ERR_UNSUPPORTED;
    return t4b::gemv_w4_decode_grouped_plan(n, N, M, K, group_size, has_zero_points != 0, ctas);
}

int t4b_set_gemv_kernel(int which) {
    if (which != T4B_GEMV_AUTO && which != T4B_GEMV_GENERIC && which != T4B_GEMV_STREAM && which != T4B_GEMV_TC_SINGLE)
        return -1;
    return t4b::g_gemv_kernel.exchange(which);
}

int t4b_fused_w4a16_gemm_u4(const void* A, const void* W_packed, const void* scales, const void* zero_points,
                            void* C, int M, int N, int K, int group_size, void* stream) {
    return t4b::fused_gemm<false>(A, W_packed, scales, zero_points, C, M, N, K, group_size, stream);
}

int t4b_fused_w4a16_gemm_s4(const void* A, const void* W_packed, const void* scales, const void* zero_points,
                            void* C, int M, int N, int K, int group_size, void* stream) {
    return t4b::fused_gemm<true>(A, W_packed, scales, zero_points, C, M, N, K, group_size, stream);
}

int t4b_fused_w4a16_gemv_allgather_supported(int M, int N, int K, int group_size, int has_zero_points) {
    if (M < 1 || N < 1 || K < 8 || (K % 8) != 0) return T4B_ERR_INVALID_VALUE;
    if (group_size < 8 || (group_size % 8) != 0 || (K % group_size) != 0) return T4B_ERR_INVALID_VALUE;
    if (N & 1) return T4B_ERR_UNSUPPORTED;       // whole column pairs
    return t4b::gemv_w4_decode_supported(M, N, K, group_size, has_zero_points != 0);
}

int t4b_fused_w4a16_gemv_allgather_grouped(const void* A, int n, const void* const* W_packed,
                                           const void* const* scales, const void* const* zero_points, const int* N,
                                           const int* col_offsets, int M, int K, int group_size, int is_signed,
                                           const T4BGather* gather, void* stream) {
    if (n < 1 || n > T4B_GROUPED_MAX || M < 1 || K < 8 || (K % 8) != 0) return T4B_ERR_INVALID_VALUE;
    if (group_size < 8 || (group_size % 8) != 0 || (K % group_size) != 0) return T4B_ERR_INVALID_VALUE;
    if (!A || !W_packed || !scales || !N || !col_offsets || !gather) return T4B_ERR_NULL_POINTER;
    for (int j = 0; j < n; ++j) {
        if (N[j] < 1) return T4B_ERR_INVALID_VALUE;
        if (!W_packed[j] || !scales[j] || (zero_points && !zero_points[j])) return T4B_ERR_NULL_POINTER;
    }
    return t4b::gemv_w4_decode_gather_grouped(is_signed != 0, A, n, W_packed, scales, zero_points, N, col_offsets, M,
                                              K, group_size, gather, static_cast<cudaStream_t>(stream));
}

int t4b_fused_w4a16_gemv_allgather(const void* A, const void* W_packed, const void* scales, const void* zero_points,
                                   int M, int N, int K, int group_size, int is_signed, const T4BGather* gather,
                                   void* stream) {
    if (M < 1 || N < 1 || K < 8 || (K % 8) != 0) return T4B_ERR_INVALID_VALUE;
    if (group_size < 8 || (group_size % 8) != 0 || (K % group_size) != 0) return T4B_ERR_INVALID_VALUE;
    if (!A || !W_packed || !scales || !gather) return T4B_ERR_NULL_POINTER;
    return t4b::gemv_w4_decode_gather(is_signed != 0, A, W_packed, scales, zero_points, M, N, K, group_size, gather,
                                      static_cast<cudaStream_t>(stream));
}

}  // extern "C"
