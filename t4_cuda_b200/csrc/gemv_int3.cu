// H17 fused INT3 GEMV:  C[M, N] = A[M, K] x dequant_s3(W)[K, N].
//
// Replaces src/kernels/h17_mega_kernel.cu:24-141 (scalar 4-byte loads, 64
// threads per column, group fixed at 100).  Same skeleton as the W4A16 GEMV
// (gemv_w4.cu): a warp owns 64 columns, 128-bit word loads, register dequant
// into exact fp16 weights that feed mma.m16n8k16 as its A fragment, K split
// over warps and over a thread-block cluster reduced through DSMEM.
//
// INT3 specifics:
//  * A step covers 8 word rows (80 K); lane c takes rows kw0 + 2c and
//    kw0 + 2c + 1, i.e. 20 consecutive K, which is 5 MMAs of K = 16 per tile.
//  * unpack_s3_exact (common.cuh) yields pairs (e_i, e_{i+5}); the activation
//    fragment is permuted to the same pairs with PRMTs.
//  * Any group size >= 10 works.  When a word straddles a group boundary (group 128:
//    10*kw .. 10*kw+9 crosses a multiple of 128) each pair picks its scale and
//    zero point per element; otherwise one scale serves the whole word.
#include "common.cuh"
#include "tma.cuh"

#include <atomic>
#include <cooperative_groups.h>

namespace cg = cooperative_groups;

namespace t4b {
namespace {

constexpr int kWarps = 8;

// 0: register streaming (the default); 1: the warp-specialized TMA-ring form
// where it applies; 2: register streaming at every M (0 and 1 run M > 16 on
// the tcgen05 GEMM where it takes the shape); 3: the tcgen05 GEMM at every M
// where it takes the shape.  The ring form is correct and tested but slower on every
// benchmarked shape (14340 x 14336: 99 against 63 us): the step math -- ~9
// integer and ~10 fp16 operations per 10-weight word for the exact contract
// dequant with per-element group selection -- bounds this kernel, not the
// weight stream, and the register-streaming form keeps more steps in flight
// per SM (16 warps with two steps each against 8 warps with one).
std::atomic<int> g_int3_kernel{0};
constexpr int kTileN = 64;
constexpr int kNB = 2;

// CTAs per SM the register budget is sized for.  The kernel is latency-bound
// (a warp's dequant + MMA chain per step), so warps per SM matter more than
// registers: the M <= 8, no-zero-point form fits two CTAs (128 registers, a
// few bytes of spill); the others need ~170-240 registers and stay at one.
template <int MT, bool HAS_ZP>
constexpr int min_blocks() { return (MT == 1 && !HAS_ZP) ? 2 : 1; }

struct Int3Params {
    const uint16_t* A;       // [M, K]
    const uint32_t* W;       // [K/10, N]
    const uint16_t* S;       // [G, N]
    const uint16_t* Z;       // [G, N] or null
    uint16_t* C;             // [M, N]
    int M, N, K, KW, G;      // KW = K / 10, G = number of groups
    int group;               // elements per group
    FastDiv gdiv;            // division by group
    int steps_per_warp;
    int total_steps;         // ceil(KW / 8)
    int a_vec8;              // activation rows are 8-byte aligned (K % 4 == 0)
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

__device__ __forceinline__ int slot_col(int r, int j) { return (j < 4) ? 4 * r + j : 32 + 4 * r + (j - 4); }

template <int MT, bool HAS_ZP>
struct Int3Step {
    uint32_t w[2][8];        // [row e][slot j]
    uint32_t slo[2][4];      // scales of the word's first group, fp16 pairs of slots (2i, 2i+1)
    uint32_t shi[2][4];      // scales of the next group (used when the word straddles)
    uint32_t zlo[2][HAS_ZP ? 4 : 1];
    uint32_t zhi[2][HAS_ZP ? 4 : 1];
    int split[2];            // first element index in the next group (10 = no straddle)
    uint32_t a[MT][10];      // 20 activations of row m0 + 8 mt + r at K = 10 (kw0 + 2c)
};

template <bool VEC>
__device__ __forceinline__ void load_row4(const uint16_t* base, size_t off, int col, int N, bool v, uint32_t& x0,
                                          uint32_t& x1) {
    if (VEC) {
        const uint2 t = v ? __ldg(reinterpret_cast<const uint2*>(base + off)) : make_uint2(0, 0);
        x0 = t.x; x1 = t.y;
    } else {
        uint16_t h[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) h[j] = (v && col + j < N) ? __ldg(base + off + j) : (uint16_t)0;
        x0 = h2_pack(h[0], h[1]); x1 = h2_pack(h[2], h[3]);
    }
}

template <int MT, bool HAS_ZP, bool VEC>
__device__ __forceinline__ void load_step(const Int3Params& p, Int3Step<MT, HAS_ZP>& d, int step, bool in_range,
                                          int r, int c, int n0, int m0) {
    const int kwb = 8 * step + 2 * c;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        const int kw = kwb + e;
        const bool vk = in_range && kw < p.KW;
        const int k0 = 10 * kw;
        const int g = vk ? (int)fdiv((uint32_t)k0, p.gdiv) : 0;
        const int split = (g + 1) * p.group - k0;          // elements >= split use group g + 1
        const bool straddle = vk && split < 10;
        d.split[e] = straddle ? split : 10;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int col = n0 + 32 * h + 4 * r;
            const bool v = vk && col < p.N;
            if (VEC) {
                const uint4 wv = v ? ld_stream(p.W + (size_t)kw * p.N + col) : make_uint4(0, 0, 0, 0);
                d.w[e][4 * h + 0] = wv.x; d.w[e][4 * h + 1] = wv.y; d.w[e][4 * h + 2] = wv.z; d.w[e][4 * h + 3] = wv.w;
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    d.w[e][4 * h + j] = (v && col + j < p.N) ? __ldg(p.W + (size_t)kw * p.N + col + j) : 0u;
            }
            load_row4<VEC>(p.S, (size_t)g * p.N + col, col, p.N, v, d.slo[e][2 * h], d.slo[e][2 * h + 1]);
            load_row4<VEC>(p.S, (size_t)(g + 1) * p.N + col, col, p.N, v && straddle, d.shi[e][2 * h], d.shi[e][2 * h + 1]);
            if constexpr (HAS_ZP) {
                load_row4<VEC>(p.Z, (size_t)g * p.N + col, col, p.N, v, d.zlo[e][2 * h], d.zlo[e][2 * h + 1]);
                load_row4<VEC>(p.Z, (size_t)(g + 1) * p.N + col, col, p.N, v && straddle, d.zhi[e][2 * h],
                               d.zhi[e][2 * h + 1]);
            }
        }
    }
    const bool vk0 = in_range && kwb < p.KW;
    const bool vk1 = in_range && kwb + 1 < p.KW;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
        const int m = m0 + 8 * mt + r;
        const uint16_t* src = p.A + (size_t)m * p.K + 10 * kwb;
        const bool vm = m < p.M;
        if (p.a_vec8) {
            // halves 0..9 belong to word kwb, 10..19 to word kwb + 1; the middle
            // 8-byte vector (halves 8..11) straddles them and is read whole only
            // when both words are inside K.
#pragma unroll
            for (int q = 0; q < 5; ++q) {
                uint32_t lo = 0u, hi = 0u;
                if (q == 2) {
                    if (vm && vk1) {
                        const uint2 t = __ldg(reinterpret_cast<const uint2*>(src) + q);
                        lo = t.x; hi = t.y;
                    } else if (vm && vk0) {
                        lo = __ldg(reinterpret_cast<const uint32_t*>(src) + 4);
                    }
                } else if (vm && (q < 2 ? vk0 : vk1)) {
                    const uint2 t = __ldg(reinterpret_cast<const uint2*>(src) + q);
                    lo = t.x; hi = t.y;
                }
                d.a[mt][2 * q] = lo; d.a[mt][2 * q + 1] = hi;
            }
        } else {
#pragma unroll
            for (int q = 0; q < 10; ++q) {
                const bool v = vm && (q < 5 ? vk0 : vk1);
                d.a[mt][q] = v ? __ldg(reinterpret_cast<const uint32_t*>(src) + q) : 0u;
            }
        }
    }
}

// Scale (and zero-point) pair for element pair (i, i+5) of slot j when the word
// straddles: element x uses the next group iff x >= split.
__device__ __forceinline__ uint32_t pick_pair(uint32_t lo_pair2, uint32_t hi_pair2, int j, int i, int split) {
    const uint16_t lo = (j & 1) ? (uint16_t)(lo_pair2 >> 16) : (uint16_t)(lo_pair2 & 0xFFFF);
    const uint16_t hi = (j & 1) ? (uint16_t)(hi_pair2 >> 16) : (uint16_t)(hi_pair2 & 0xFFFF);
    return h2_pack(i >= split ? hi : lo, (i + 5) >= split ? hi : lo);
}

template <int MT, bool HAS_ZP>
__device__ __forceinline__ void compute_step(const Int3Step<MT, HAS_ZP>& d, float (&acc)[MT][4][4]) {
    // activation pairs: index 5e + i -> (a[10e + i], a[10e + i + 5])
    uint32_t b[MT][10];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const uint32_t* x = &d.a[mt][5 * e];
            b[mt][5 * e + 0] = prmt(x[0], x[2], 0x7610);
            b[mt][5 * e + 1] = prmt(x[0], x[3], 0x5432);
            b[mt][5 * e + 2] = prmt(x[1], x[3], 0x7610);
            b[mt][5 * e + 3] = prmt(x[1], x[4], 0x5432);
            b[mt][5 * e + 4] = prmt(x[2], x[4], 0x7610);
        }
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        uint32_t Q[2][10];   // [row r / r+8][5 e + i]
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            const int j = 2 * t + rr;
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                uint32_t q[5];
                unpack_s3_exact(d.w[e][j], q);
                if (d.split[e] >= 10) {
                    const uint32_t sp = d.slo[e][j >> 1];
                    const uint32_t s2 = prmt(sp, sp, (j & 1) ? 0x3232 : 0x1010);
                    uint32_t z2 = 0;
                    if constexpr (HAS_ZP) {
                        const uint32_t zp = d.zlo[e][j >> 1];
                        z2 = prmt(zp, zp, (j & 1) ? 0x3232 : 0x1010);
                    }
#pragma unroll
                    for (int i = 0; i < 5; ++i) Q[rr][5 * e + i] = h2_mul(HAS_ZP ? h2_sub(q[i], z2) : q[i], s2);
                } else {
#pragma unroll
                    for (int i = 0; i < 5; ++i) {
                        const uint32_t s2 = pick_pair(d.slo[e][j >> 1], d.shi[e][j >> 1], j, i, d.split[e]);
                        uint32_t qi = q[i];
                        if constexpr (HAS_ZP)
                            qi = h2_sub(qi, pick_pair(d.zlo[e][j >> 1], d.zhi[e][j >> 1], j, i, d.split[e]));
                        Q[rr][5 * e + i] = h2_mul(qi, s2);
                    }
                }
            }
        }
#pragma unroll
        for (int u = 0; u < 5; ++u)
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
                mma_16816(acc[mt][t], Q[0][2 * u], Q[1][2 * u], Q[0][2 * u + 1], Q[1][2 * u + 1], b[mt][2 * u],
                          b[mt][2 * u + 1]);
    }
}

template <int MT, bool HAS_ZP, bool VEC, bool CLUSTER>
__global__ void __launch_bounds__(kWarps * 32, min_blocks<MT, HAS_ZP>())
gemv_int3_kernel(const Int3Params p) {
    constexpr int MR = 8 * MT;
    constexpr int RED_STRIDE = MR + 1;
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

    // programmatic dependent launch: the next kernel may start as SMs free up;
    // this one reads A and writes C only after the previous kernel is done
    pdl_launch_dependents();
    pdl_wait_prior_grid();
    Int3Step<MT, HAS_ZP> buf[kNB];
#pragma unroll
    for (int i = 0; i < kNB; ++i)
        load_step<MT, HAS_ZP, VEC>(p, buf[i], s_begin + i, s_begin + i < s_end, r, c, n0, m0);
    for (int s = s_begin; s < s_end; s += kNB) {
#pragma unroll
        for (int i = 0; i < kNB; ++i) {
            if (s + i < s_end) {
                compute_step<MT, HAS_ZP>(buf[i], acc);
                const int nxt = s + i + kNB;
                load_step<MT, HAS_ZP, VEC>(p, buf[i], nxt, nxt < s_end, r, c, n0, m0);
            }
        }
    }

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
        cluster.sync();
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

// ---------------------------------------------------------------------------
// Warp-specialized TMA-ring form (selected by t4b_set_int3_kernel).  The same
// step math as above, but the words reach the math warps through a ring of
// shared-memory stages that one producer warp fills with TMA: every stage the
// ring holds is requested at kernel entry, before griddepcontrol.wait, so the
// weight stream of a CTA's K range is in flight while the previous kernel
// drains, and a math warp's step waits on shared memory (~30 cycles), not on
// HBM.  A stage is 64 word rows (one 8-row step per math warp) of the CTA's 64
// columns, two 32-column boxes with 128-byte swizzle: lane (r, c) reads rows
// 2c and 2c + 1 of its warp's 8 at 16-byte unit r ^ (row & 7), which puts the
// 8 lanes of every quarter-warp on 8 distinct bank groups.  Scales, zero points
// and activations are read as in the register-streaming form (they are small
// and cached).  K is split over a cluster exactly as there.
namespace ring {

constexpr int kRows = 8 * kWarps;                       // word rows per stage
constexpr int kBoxCols = 32;                            // 128-byte box rows
constexpr int kStageBytes = kRows * kTileN * 4;         // 16 KB
constexpr int kMaxStages = 12;
constexpr int kThreads = (kWarps + 1) * 32;             // + one producer warp
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr unsigned kErrTimeout = 1u;

// Device error word of the ring form (bit 0: a bounded wait gave up).
__device__ unsigned g_int3_error = 0;

struct RingParams {
    int stages;           // ring depth
    int rows_per_split;   // word rows of one K split (a multiple of 8)
    int total_steps;      // 8-row steps of the whole K (ceil(KW / 8))
};

// The words of `step` (8-row step of the whole K) for this lane from ring
// slot `slot_a` (row 8 * warp + 2c + e of the stage), plus its scales, zero
// points and activations as load_step reads them.
template <int MT, bool HAS_ZP>
__device__ __forceinline__ void load_step_smem(const Int3Params& p, Int3Step<MT, HAS_ZP>& d, uint32_t slot_a, int step,
                                               bool in_range, int warp, int r, int c, int n0, int m0) {
    const int kwb = 8 * step + 2 * c;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        const int kw = kwb + e;
        const bool vk = in_range && kw < p.KW;
        const int k0 = 10 * kw;
        const int g = vk ? (int)fdiv((uint32_t)k0, p.gdiv) : 0;
        const int split = (g + 1) * p.group - k0;          // elements >= split use group g + 1
        const bool straddle = vk && split < 10;
        d.split[e] = straddle ? split : 10;
        const int row = 8 * warp + 2 * c + e;              // row within the stage
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int col = n0 + 32 * h + 4 * r;
            const bool v = vk && col < p.N;
            uint4 wv = make_uint4(0, 0, 0, 0);
            if (vk) {
                const uint32_t a = slot_a + (uint32_t)(h * (kRows * 128) + row * 128) + (uint32_t)((r ^ (row & 7)) << 4);
                asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                             : "=r"(wv.x), "=r"(wv.y), "=r"(wv.z), "=r"(wv.w) : "r"(a) : "memory");
            }
            d.w[e][4 * h + 0] = wv.x; d.w[e][4 * h + 1] = wv.y; d.w[e][4 * h + 2] = wv.z; d.w[e][4 * h + 3] = wv.w;
            load_row4<true>(p.S, (size_t)g * p.N + col, col, p.N, v, d.slo[e][2 * h], d.slo[e][2 * h + 1]);
            load_row4<true>(p.S, (size_t)(g + 1) * p.N + col, col, p.N, v && straddle, d.shi[e][2 * h], d.shi[e][2 * h + 1]);
            if constexpr (HAS_ZP) {
                load_row4<true>(p.Z, (size_t)g * p.N + col, col, p.N, v, d.zlo[e][2 * h], d.zlo[e][2 * h + 1]);
                load_row4<true>(p.Z, (size_t)(g + 1) * p.N + col, col, p.N, v && straddle, d.zhi[e][2 * h],
                                d.zhi[e][2 * h + 1]);
            }
        }
    }
    const bool vk0 = in_range && kwb < p.KW;
    const bool vk1 = in_range && kwb + 1 < p.KW;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
        const int m = m0 + 8 * mt + r;
        const uint16_t* src = p.A + (size_t)m * p.K + 10 * kwb;
        const bool vm = m < p.M;
        if (p.a_vec8) {
#pragma unroll
            for (int q = 0; q < 5; ++q) {
                uint32_t lo = 0u, hi = 0u;
                if (q == 2) {
                    if (vm && vk1) {
                        const uint2 t = __ldcg(reinterpret_cast<const uint2*>(src) + q);
                        lo = t.x; hi = t.y;
                    } else if (vm && vk0) {
                        lo = __ldcg(reinterpret_cast<const uint32_t*>(src) + 4);
                    }
                } else if (vm && (q < 2 ? vk0 : vk1)) {
                    const uint2 t = __ldcg(reinterpret_cast<const uint2*>(src) + q);
                    lo = t.x; hi = t.y;
                }
                d.a[mt][2 * q] = lo; d.a[mt][2 * q + 1] = hi;
            }
        } else {
#pragma unroll
            for (int q = 0; q < 10; ++q) {
                const bool v = vm && (q < 5 ? vk0 : vk1);
                d.a[mt][q] = v ? __ldcg(reinterpret_cast<const uint32_t*>(src) + q) : 0u;
            }
        }
    }
}

template <int MT, bool HAS_ZP, bool CLUSTER>
__global__ void __launch_bounds__(kThreads, 1)
gemv_int3_ring_kernel(const __grid_constant__ CUtensorMap wmap, const Int3Params p, const RingParams rp) {
    constexpr int MR = 8 * MT;
    constexpr int RED_STRIDE = MR + 1;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    float* red = reinterpret_cast<float*>(ring + (size_t)rp.stages * kStageBytes);   // [kWarps][kTileN * RED_STRIDE]
    uint64_t* full = reinterpret_cast<uint64_t*>(red + kWarps * kTileN * RED_STRIDE);
    uint64_t* empty = full + kMaxStages;
    volatile int* sflag = reinterpret_cast<volatile int*>(empty + kMaxStages);   // [0] abort, [1] stages issued

    pdl_launch_dependents();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int n0 = blockIdx.x * kTileN;
    const int m0 = blockIdx.z * MR;
    const int kb = blockIdx.y * rp.rows_per_split;                 // first word row of this split
    const int ke = min(p.KW, kb + rp.rows_per_split);
    const int nst = ke > kb ? (ke - kb + kRows - 1) / kRows : 0;   // stages of this CTA
    if (threadIdx.x == 0) {
        for (int s = 0; s < rp.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kWarps);
        }
        sflag[0] = 0;
        sflag[1] = 0;
        fence_barrier_init();
    }
    __syncthreads();

    float acc[MT][4][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int t = 0; t < 4; ++t)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[mt][t][i] = 0.f;

    if (warp == kWarps) {
        // ---------------- producer: every stage the ring holds before the
        // dependency wait (the words are never written by a kernel of this
        // library), then refills as the math warps release slots
        if (lane == 0) {
            prefetch_tmap(&wmap);
            auto issue = [&](int i, int slot) {
                uint8_t* dst = ring + (size_t)slot * kStageBytes;
                mbar_arrive_expect_tx(&full[slot], (uint32_t)kStageBytes);
                tma_load_2d(dst, &wmap, n0, kb + i * kRows, &full[slot]);
                tma_load_2d(dst + kRows * 128, &wmap, n0 + kBoxCols, kb + i * kRows, &full[slot]);
            };
            const int early = nst < rp.stages ? nst : rp.stages;
            for (int i = 0; i < early; ++i) issue(i, i);
            sflag[1] = early;
            bool ok = true;
            for (int i = early; i < nst; ++i) {
                const int slot = i % rp.stages;
                if (!mbar_wait_bounded(&empty[slot], (uint32_t)(((i / rp.stages) & 1) ^ 1), kWaitLimitNs)) {
                    ok = false;
                    break;
                }
                if (sflag[0]) break;
                fence_proxy_async_smem();    // the math warps' reads of the slot before the copy overwrites it
                issue(i, slot);
                sflag[1] = i + 1;
            }
            if (!ok) {
                sflag[0] = 1;
                atomicOr(&g_int3_error, kErrTimeout);
            }
        }
    } else {
        // ---------------- math warps: one 8-row step per stage each
        const int r = lane >> 2, c = lane & 3;
        pdl_wait_prior_grid();       // A may belong to the previous kernel
        const uint32_t ring_a = smem_addr(ring);
        bool aborted = false;
        Int3Step<MT, HAS_ZP> d;
        for (int i = 0; i < nst; ++i) {
            const int slot = i % rp.stages;
            if (!aborted && sflag[0]) aborted = true;      // the producer gave up: nothing more lands
            if (!aborted && !mbar_wait_bounded(&full[slot], (uint32_t)((i / rp.stages) & 1), kWaitLimitNs)) {
                aborted = true;
                sflag[0] = 1;
                atomicOr(&g_int3_error, kErrTimeout);
            }
            const int step = (kb >> 3) + i * kWarps + warp;
            const bool in_range = !aborted && 8 * step < ke;
            load_step_smem<MT, HAS_ZP>(p, d, ring_a + (uint32_t)slot * kStageBytes, step, in_range, warp, r, c, n0, m0);
            // the slot's words are in registers: release it before the math
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (in_range) compute_step<MT, HAS_ZP>(d, acc);
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const int c0 = slot_col(r, 2 * t), c1 = slot_col(r, 2 * t + 1);
                const int mm = 8 * mt + 2 * c;
                float* rw = red + warp * (kTileN * RED_STRIDE);
                rw[c0 * RED_STRIDE + mm] = acc[mt][t][0];
                rw[c0 * RED_STRIDE + mm + 1] = acc[mt][t][1];
                rw[c1 * RED_STRIDE + mm] = acc[mt][t][2];
                rw[c1 * RED_STRIDE + mm + 1] = acc[mt][t][3];
            }
    }
    __syncthreads();
    if (sflag[0] && threadIdx.x == 0) {
        // do not leave while copies may still be landing in this CTA's memory
        const int issued = sflag[1];
        for (int j = (issued > rp.stages ? issued - rp.stages : 0); j < issued; ++j)
            mbar_wait_bounded(&full[j % rp.stages], (uint32_t)((j / rp.stages) & 1), kWaitLimitNs / 4);
    }
    constexpr int OUTS = kTileN * MR;
    for (int o = threadIdx.x; o < OUTS; o += kThreads) {
        const int idx = (o / MR) * RED_STRIDE + (o % MR);
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) v += red[w * (kTileN * RED_STRIDE) + idx];
        red[idx] = v;
    }
    if constexpr (CLUSTER) {
        cg::cluster_group cluster = cg::this_cluster();
        cluster.sync();
        const int nranks = (int)cluster.num_blocks();
        const int rank = (int)cluster.block_rank();
        const int per = (OUTS + nranks - 1) / nranks;
        const int o_end = min(OUTS, (rank + 1) * per);
        for (int o = rank * per + threadIdx.x; o < o_end; o += kThreads) {
            const int col = o / MR, mm = o % MR;
            const int idx = col * RED_STRIDE + mm;
            float v = 0.f;
            for (int q = 0; q < nranks; ++q) v += cluster.map_shared_rank(red, q)[idx];
            const int m = m0 + mm, n = n0 + col;
            if (m < p.M && n < p.N) p.C[(size_t)m * p.N + n] = __half_as_ushort(__float2half_rn(v));
        }
        cluster.sync();
    } else {
        __syncthreads();
        for (int o = threadIdx.x; o < OUTS; o += kThreads) {
            const int col = o / MR, mm = o % MR;
            const int m = m0 + mm, n = n0 + col;
            if (m < p.M && n < p.N) p.C[(size_t)m * p.N + n] = __half_as_ushort(__float2half_rn(red[col * RED_STRIDE + mm]));
        }
    }
}

template <int MT, bool HAS_ZP>
int launch(const CUtensorMap& wmap, const Int3Params& p, const RingParams& rp, int splits, size_t smem,
           cudaStream_t stream) {
    auto kern = splits > 1 ? gemv_int3_ring_kernel<MT, HAS_ZP, true> : gemv_int3_ring_kernel<MT, HAS_ZP, false>;
    static SmemLimit limit[2];     // per instantiation (cluster or not), per device
    const int st = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), (int)smem, &limit[splits > 1 ? 1 : 0]);
    if (st != T4B_OK) return st;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((p.N + kTileN - 1) / kTileN, splits, (p.M + 8 * MT - 1) / (8 * MT));
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int n = 0;
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
    if (splits > 1) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = 1;
        attr[n].val.clusterDim.y = splits;
        attr[n].val.clusterDim.z = 1;
        ++n;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    cudaError_t err = cudaLaunchKernelEx(&cfg, kern, wmap, p, rp);
    if (err != cudaSuccess) return record_cuda_error(err);
    return T4B_OK;
}

// T4B_ERR_UNSUPPORTED (nothing launched) where the ring form does not apply.
int fused_int3_ring(const Int3Params& p, const void* W, cudaStream_t stream) {
    if ((p.N % 4) != 0 || !aligned(W, 16) || !aligned(p.S, 8) || (p.Z && !aligned(p.Z, 8))) return T4B_ERR_UNSUPPORTED;
    const int mt = (p.M <= 8) ? 1 : 2;
    const int tiles = (p.N + kTileN - 1) / kTileN;
    const int chunks = (p.M + 8 * mt - 1) / (8 * mt);
    // split K over a cluster until the CTAs cover the SMs, at most 8 ways, and
    // at least one stage each
    int splits = sm_count() / (tiles * chunks);
    if (splits > 8) splits = 8;
    while (splits > 1 && splits * kRows > p.KW) --splits;
    if (splits < 1) splits = 1;
    while (splits > 1 && (splits & (splits - 1))) --splits;   // cluster sizes 1, 2, 4, 8
    RingParams rp;
    rp.total_steps = (p.KW + 7) / 8;
    rp.rows_per_split = 8 * ((rp.total_steps + splits - 1) / splits);
    const size_t red_bytes = (size_t)kWarps * kTileN * (8 * mt + 1) * 4;
    const size_t fixed = 1024 + red_bytes + 2 * kMaxStages * 8 + 16;
    int optin = 0, per_sm = 0, reserved = 0, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev);
    // more CTAs than SMs (wide N): a ring half the size so that two CTAs share
    // an SM and the grid runs as one wave
    const bool two_per_sm = tiles * chunks * splits > sm_count();
    const size_t budget = two_per_sm ? (size_t)(per_sm / 2 - reserved) : (size_t)optin;
    int stages = budget > fixed ? (int)((budget - fixed) / kStageBytes) : 0;
    if (stages > kMaxStages) stages = kMaxStages;
    if (stages < 2) return T4B_ERR_UNSUPPORTED;
    rp.stages = stages;
    const size_t smem = fixed + (size_t)stages * kStageBytes;
    CUtensorMap wmap;
    if (!make_tmap_2d_ex(&wmap, false, W, (uint64_t)p.KW, (uint64_t)p.N, kRows, kBoxCols, 128, 256))
        return T4B_ERR_UNSUPPORTED;
    const bool zp = p.Z != nullptr;
    if (mt == 1) return zp ? launch<1, true>(wmap, p, rp, splits, smem, stream) : launch<1, false>(wmap, p, rp, splits, smem, stream);
    return zp ? launch<2, true>(wmap, p, rp, splits, smem, stream) : launch<2, false>(wmap, p, rp, splits, smem, stream);
}

}  // namespace ring

template <int MT, bool HAS_ZP, bool VEC>
int launch(const Int3Params& p, int splits, cudaStream_t stream) {
    const dim3 block(kWarps * 32);
    const dim3 grid((p.N + kTileN - 1) / kTileN, splits, (p.M + 8 * MT - 1) / (8 * MT));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;       // K split over a cluster (DSMEM reduction)
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = splits;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = splits > 1 ? 2 : 1;
    cudaError_t err = splits > 1 ? cudaLaunchKernelEx(&cfg, gemv_int3_kernel<MT, HAS_ZP, VEC, true>, p)
                                 : cudaLaunchKernelEx(&cfg, gemv_int3_kernel<MT, HAS_ZP, VEC, false>, p);
    if (err != cudaSuccess) return record_cuda_error(err);
    return check_launch();
}

template <int MT, bool HAS_ZP>
int dispatch_vec(const Int3Params& p, bool vec, int splits, cudaStream_t s) {
    return vec ? launch<MT, HAS_ZP, true>(p, splits, s) : launch<MT, HAS_ZP, false>(p, splits, s);
}

int fused_int3(const void* A, const void* W, const void* S, const void* Z, void* C, int M, int N, int K, int group,
               void* stream_) {
    if (M < 1 || N < 1 || K < 10 || (K % 10) != 0 || group < 1) return T4B_ERR_INVALID_VALUE;
    // a 10-element word may straddle at most one group boundary
    if (group < 10) return T4B_ERR_UNSUPPORTED;
    if (!A || !W || !S || !C) return T4B_ERR_NULL_POINTER;
    if (!aligned(A, 16) || !aligned(W, 4) || !aligned(S, 2) || !aligned(C, 2) || (Z && !aligned(Z, 2)))
        return T4B_ERR_MISALIGNED;
    Int3Params p;
    p.A = static_cast<const uint16_t*>(A);
    p.W = static_cast<const uint32_t*>(W);
    p.S = static_cast<const uint16_t*>(S);
    p.Z = static_cast<const uint16_t*>(Z);
    p.C = static_cast<uint16_t*>(C);
    p.M = M; p.N = N; p.K = K; p.KW = K / 10;
    p.group = group;
    p.G = (K + group - 1) / group;
    p.gdiv = make_fastdiv((uint32_t)group);
    p.total_steps = (p.KW + 7) / 8;
    p.a_vec8 = (K % 4 == 0) ? 1 : 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream_);
    const int choice = g_int3_kernel.load();
    // M > 16: the tcgen05 GEMM where it takes the shape
    if ((M > 16 && choice != 2) || choice == 3) {
        const int st = gemm_int3_tc(A, W, S, Z, C, M, N, K, group, choice == 3, s);
        if (st != T4B_ERR_UNSUPPORTED) return st;
    }
    if (choice == 1) {
        const int st = ring::fused_int3_ring(p, W, s);
        if (st != T4B_ERR_UNSUPPORTED) return st;
    }
    const bool vec = (N % 4 == 0) && aligned(W, 16) && aligned(S, 8) && (!Z || aligned(Z, 8));
    const int mt = (M <= 8) ? 1 : 2;
    const int tiles = (N + kTileN - 1) / kTileN;
    const int chunks = (M + 8 * mt - 1) / (8 * mt);
    // Split K only as far as one wave of CTAs covers the SMs (min_blocks per
    // SM): a second wave would repeat the whole load round trip.
    const int per_sm = (mt == 1 && !Z) ? min_blocks<1, false>() : 1;
    int splits = per_sm * sm_count() / (tiles * chunks);
    if (splits > 8) splits = 8;
    while (splits > 1 && splits * kWarps > p.total_steps) --splits;
    if (splits < 1) splits = 1;
    const int warps = splits * kWarps;
    p.steps_per_warp = (p.total_steps + warps - 1) / warps;
    if (mt == 1) return Z ? dispatch_vec<1, true>(p, vec, splits, s) : dispatch_vec<1, false>(p, vec, splits, s);
    return Z ? dispatch_vec<2, true>(p, vec, splits, s) : dispatch_vec<2, false>(p, vec, splits, s);
}

}  // namespace

int int3_device_error(cudaStream_t stream, unsigned* out, bool clear) {
    unsigned* word = nullptr;
    cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&word), ring::g_int3_error);
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, word, sizeof(unsigned), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess && clear) e = cudaMemsetAsync(word, 0, sizeof(unsigned), stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    return e == cudaSuccess ? T4B_OK : record_cuda_error(e);
}

}  // namespace t4b

extern "C" int t4b_set_int3_kernel(int which) {
    if (which < 0 || which > 3) return -1;
    return t4b::g_int3_kernel.exchange(which);
}

extern "C" int t4b_fused_h17_gemv_s3(const void* A, const void* W_packed, const void* scales,
                                     const void* zero_points, void* C, int M, int N, int K, int group_size,
                                     void* stream) {
    return t4b::fused_int3(A, W_packed, scales, zero_points, C, M, N, K, group_size, stream);
}
