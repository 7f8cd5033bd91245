// Decode GEMV / skinny GEMM that streams the packed weights with TMA, balanced
// over all SMs ("stream-K"), and overlaps consecutive launches.
//
//   C[M, N] = A[M, K] x dequant(W)[K, N],  W int32 [K/8, N], group scales [K/g, N]
//
// Work decomposition
//   The weight matrix is cut into chunks of 64 word rows x 64 columns (16 KB).
//   Chunks are numbered tile-major (column tile t, K chunk kc fastest) and the
//   grid of one CTA per SM takes equal contiguous runs of them, so every SM
//   streams the same number of bytes whatever the shape.  A CTA's run covers
//   one to a few column tiles; a tile split between CTAs is finished by the
//   last of them (fixed-order sum of the per-CTA partials in a workspace,
//   counters reset by that CTA), so results are deterministic.
//
// Pipeline (8 warps, no dedicated producer)
//   Chunks arrive by TMA as two 32-column x 64-row boxes with 128-byte swizzle
//   in a 4-deep shared-memory ring, completion signalled on an mbarrier.
//   Thread 0 issues the first four chunks at kernel entry -- before
//   griddepcontrol.wait, because packed weights are never written by a kernel
//   of this library -- so under programmatic dependent launch a GEMV's
//   weights stream in while the previous kernel is still running.  A CTA is
//   small enough (256 threads, <= 128 registers, ~83 KB shared memory) for two
//   to share an SM, which is what lets the next launch start early.  Whichever
//   warp finishes a slot last (shared-memory counter) refills it.
//
// Math per warp and chunk
//   Warp w owns word rows 8w..8w+7: two MMA steps of 4 rows x 64 columns.
//   Lane (r, c) reads row 8w + 4s + c, 16-byte chunk L(r) = r/2 + 4 (r%2) of
//   each box; with the 128-byte swizzle the eight lanes of a quarter warp hit
//   eight different bank groups.  Words become exact fp16 integers
//   (common.cuh) that are the A fragment of mma.m16n8k16 (16 output columns
//   x 16 K); activations are the B fragment.  The K-group scale multiplies the
//   fp32 partial sums once per group; zero points enter through the
//   activation sums (an extra MMA with an all-ones A fragment):
//   y += s * (sum q a - z * sum a).
#include <mutex>
#include <vector>

#include "common.cuh"
#include "tma.cuh"
#include "workspace.h"

namespace t4b {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kTileN = 64;                     // output columns per tile
constexpr int kChunkRows = 64;                 // word rows per chunk (512 K)
constexpr int kStages = 4;
constexpr int kBoxCols = 32;                   // 32 words = 128 bytes = one swizzle row
constexpr int kBoxBytes = kChunkRows * kBoxCols * 4;
constexpr int kStageBytes = 2 * kBoxBytes;
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr unsigned kErrTimeout = 1u;

struct StreamParams {
    const uint16_t* A;
    const uint16_t* S;
    const uint16_t* Z;
    uint16_t* C;
    float* part;             // [tiles][max_segs][64 * MR] partial sums of split tiles
    unsigned* flags;         // [tiles][max_segs] segment published (zero between launches)
    unsigned* err;
    int M, N, K, KW;
    int tiles, cpt, G, max_segs;
    int total;               // tiles * cpt
    FastDiv gdiv;            // division by group_size / 8
    FastDiv cdiv;            // division by cpt
};

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}

// Column of the 64-column tile held by word slot j (0..7) of a lane whose
// 16-byte box chunk is L: slots 0..3 are box 0, slots 4..7 box 1.
__device__ __forceinline__ int slot_col(int L, int j) { return 32 * (j >> 2) + 4 * L + (j & 3); }

__device__ __forceinline__ int chunk_start(int b, int total, int G) { return (int)((long long)b * total / G); }

// The CTA whose run contains chunk x.
__device__ __forceinline__ int cta_of(int x, int total, int G) {
    int b = (int)((long long)x * G / total);
    while (b + 1 < G && chunk_start(b + 1, total, G) <= x) ++b;
    while (b > 0 && chunk_start(b, total, G) > x) --b;
    return b;
}

__device__ __forceinline__ void issue_chunk(const CUtensorMap* tmap, uint8_t* ring, uint64_t* full, int slot, int t,
                                            int kc) {
    mbar_arrive_expect_tx(&full[slot], kStageBytes);
    uint8_t* dst = ring + slot * kStageBytes;
    tma_load_2d(dst, tmap, t * kTileN, kc * kChunkRows, &full[slot]);
    tma_load_2d(dst + kBoxBytes, tmap, t * kTileN + kBoxCols, kc * kChunkRows, &full[slot]);
}

template <int MT>
__device__ __forceinline__ void load_activations(const StreamParams& p, uint4 (&act)[2][MT],
                                                 const uint16_t* const (&arow)[MT], int kc, int lane_kw) {
#pragma unroll
    for (int s = 0; s < 2; ++s) {
        const int kw = kc * kChunkRows + lane_kw + 4 * s;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
            act[s][mt] = (arow[mt] && kw < p.KW) ? __ldg(reinterpret_cast<const uint4*>(arow[mt] + 8 * kw))
                                                 : make_uint4(0, 0, 0, 0);
    }
}

template <bool HAS_ZP>
__device__ __forceinline__ void load_group(const StreamParams& p, uint2 (&sp)[2], uint2 (&zp)[2], int g, int t, int L) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int col = t * kTileN + 32 * h + 4 * L;
        const bool v = col < p.N;
        sp[h] = v ? __ldg(reinterpret_cast<const uint2*>(p.S + (size_t)g * p.N + col)) : make_uint2(0, 0);
        if constexpr (HAS_ZP)
            zp[h] = v ? __ldg(reinterpret_cast<const uint2*>(p.Z + (size_t)g * p.N + col)) : make_uint2(0, 0);
    }
}

// acc += s * (dg - z * sum(a)) per column slot, then clear the group sums.
template <int MT, bool HAS_ZP>
__device__ __forceinline__ void flush_group(float (&acc)[MT][4][4], float (&dg)[MT][4][4], float (&ones)[MT][4],
                                            const uint2 (&sp)[2], const uint2 (&zp)[2]) {
    float sf[8], zf[8];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const float2 s01 = __half22float2(*reinterpret_cast<const __half2*>(&sp[h].x));
        const float2 s23 = __half22float2(*reinterpret_cast<const __half2*>(&sp[h].y));
        sf[4 * h + 0] = s01.x; sf[4 * h + 1] = s01.y; sf[4 * h + 2] = s23.x; sf[4 * h + 3] = s23.y;
        if constexpr (HAS_ZP) {
            const float2 z01 = __half22float2(*reinterpret_cast<const __half2*>(&zp[h].x));
            const float2 z23 = __half22float2(*reinterpret_cast<const __half2*>(&zp[h].y));
            zf[4 * h + 0] = z01.x; zf[4 * h + 1] = z01.y; zf[4 * h + 2] = z23.x; zf[4 * h + 3] = z23.y;
        }
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int t = 0; t < 4; ++t)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int j = 2 * t + (e >> 1);
                float v = dg[mt][t][e];
                if constexpr (HAS_ZP) v -= zf[j] * ones[mt][e & 1];
                acc[mt][t][e] = fmaf(sf[j], v, acc[mt][t][e]);
                dg[mt][t][e] = 0.f;
            }
    if constexpr (HAS_ZP) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int e = 0; e < 4; ++e) ones[mt][e] = 0.f;
    }
}

__device__ __forceinline__ void st_release_gpu(unsigned* p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Sum the 8 warps' partials of tile t in a fixed order.  A tile entirely
// inside this CTA's run is written to C; otherwise this CTA's segment is
// published: partial sums to the workspace, then a release flag.
template <int MT>
__device__ __forceinline__ void finish_tile(const StreamParams& p, float* red, float (&acc)[MT][4][4], int t,
                                            int c_begin, int c_end, int warp, int L, int c) {
    constexpr int MR = 8 * MT, RS = MR + 1, OUTS = kTileN * MR;
    const int tid = threadIdx.x;
    float* w = red + warp * kTileN * RS;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int tt = 0; tt < 4; ++tt) {
            const int c0 = slot_col(L, 2 * tt), c1 = slot_col(L, 2 * tt + 1);
            const int mm = 8 * mt + 2 * c;
            w[c0 * RS + mm] = acc[mt][tt][0];
            w[c0 * RS + mm + 1] = acc[mt][tt][1];
            w[c1 * RS + mm] = acc[mt][tt][2];
            w[c1 * RS + mm + 1] = acc[mt][tt][3];
            acc[mt][tt][0] = acc[mt][tt][1] = acc[mt][tt][2] = acc[mt][tt][3] = 0.f;
        }
    __syncthreads();
    for (int o = tid; o < OUTS; o += kThreads) {
        const int idx = (o / MR) * RS + (o % MR);
        float v = 0.f;
#pragma unroll
        for (int k = 0; k < kWarps; ++k) v += red[k * kTileN * RS + idx];
        red[idx] = v;
    }
    __syncthreads();
    const int first = t * p.cpt, last = first + p.cpt - 1;
    const int tn0 = t * kTileN;
    if (c_begin <= first && last < c_end) {
        for (int o = tid; o < OUTS; o += kThreads) {
            const int col = o / MR, mm = o % MR;
            const int n = tn0 + col;
            if (mm < p.M && n < p.N) p.C[(size_t)mm * p.N + n] = __half_as_ushort(__float2half_rn(red[col * RS + mm]));
        }
    } else {
        const int seg = blockIdx.x - cta_of(first, p.total, p.G);
        float* mine = p.part + ((size_t)t * p.max_segs + seg) * OUTS;
        for (int o = tid; o < OUTS; o += kThreads) mine[o] = red[(o / MR) * RS + (o % MR)];
        __syncthreads();   // every thread's partial store happens before thread 0's release
        if (tid == 0) st_release_gpu(&p.flags[(size_t)t * p.max_segs + seg], 1u);
    }
    __syncthreads();
}

// The CTA holding the first chunk of a split tile reduces it after its own
// run: by then the other segments were published long ago (every CTA works on
// its shared segments first).  Fixed segment order -> deterministic sums.
template <int MT>
__device__ __forceinline__ void reduce_split_tile(const StreamParams& p, int t, volatile int* sflag) {
    constexpr int MR = 8 * MT, OUTS = kTileN * MR;
    const int tid = threadIdx.x;
    const int b_first = cta_of(t * p.cpt, p.total, p.G);
    const int nseg = cta_of(t * p.cpt + p.cpt - 1, p.total, p.G) - b_first + 1;
    unsigned* flags = p.flags + (size_t)t * p.max_segs;
    if (tid == 0) {
        const uint64_t t0 = global_timer_ns();
        for (int s = 0; s < nseg; ++s) {
            while (ld_acquire_gpu(&flags[s]) == 0u) {
                if (global_timer_ns() - t0 > kWaitLimitNs) {
                    atomicOr(p.err, kErrTimeout);
                    sflag[0] = 1;
                    break;
                }
            }
        }
    }
    __syncthreads();
    const float* part = p.part + (size_t)t * p.max_segs * OUTS;
    const int tn0 = t * kTileN;
    for (int o = tid; o < OUTS; o += kThreads) {
        const int col = o / MR, mm = o % MR;
        const int n = tn0 + col;
        if (mm >= p.M || n >= p.N) continue;
        float v = 0.f;
        for (int s = 0; s < nseg; ++s) v += __ldcg(part + (size_t)s * OUTS + o);
        p.C[(size_t)mm * p.N + n] = __half_as_ushort(__float2half_rn(v));
    }
    __syncthreads();
    for (int q = tid; q < nseg; q += kThreads) flags[q] = 0u;   // ready for the next launch (it waits for this grid)
}

template <int MT>
constexpr int min_blocks() { return MT == 1 ? 2 : 1; }

template <int MT, bool SIGNED, bool HAS_ZP>
__global__ void __launch_bounds__(kThreads, min_blocks<MT>())
gemv_w4_stream_kernel(const __grid_constant__ CUtensorMap tmap, const StreamParams p) {
    constexpr int MR = 8 * MT;
    constexpr int RS = MR + 1;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* red = reinterpret_cast<float*>(ring + kStages * kStageBytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(red + kWarps * kTileN * RS);
    int* readers = reinterpret_cast<int*>(full + kStages);
    volatile int* sflag = reinterpret_cast<volatile int*>(readers + kStages);   // [0] abort, [1] last segment

    pdl_launch_dependents();
    const int b = blockIdx.x;
    const int m0 = 0;
    const int c_begin = chunk_start(b, p.total, p.G);
    const int c_end = chunk_start(b + 1, p.total, p.G);
    const int nch = c_end - c_begin;
    if (nch <= 0) return;
    // Run order: a last tile that continues into the next CTA ("shared") is
    // processed first, so its partial sums are published early; then the rest.
    const int t_first = (int)fdiv((uint32_t)c_begin, p.cdiv);
    const int t_last = (int)fdiv((uint32_t)(c_end - 1), p.cdiv);
    const bool last_shared = c_end < (t_last + 1) * p.cpt;
    const int c_split = (t_last > t_first && last_shared) ? t_last * p.cpt : c_end;
    const int n_tail = c_end - c_split;
    auto chunk_of = [&](int i) { return i < n_tail ? c_split + i : c_begin + (i - n_tail); };
    // this CTA reduces its last tile when that tile starts inside its run and is shared
    const bool reducer = last_shared && t_last * p.cpt >= c_begin;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            readers[s] = 0;
        }
        sflag[0] = 0;
        sflag[1] = 0;
        fence_barrier_init();
        prefetch_tmap(&tmap);
        // the first chunks: weights only, safe before waiting on the previous kernel
        for (int j = 0; j < kStages && j < nch; ++j) {
            const int cj = chunk_of(j);
            const int tj = (int)fdiv((uint32_t)cj, p.cdiv);
            issue_chunk(&tmap, ring, full, j, tj, cj - tj * p.cpt);
        }
    }
    __syncthreads();
    pdl_wait_prior_grid();     // A, scales, zero points, C and the workspace may belong to the previous kernel

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = lane >> 2, c = lane & 3;
    const int L = (r >> 1) + 4 * (r & 1);
    // shared-memory offsets of this lane's four 16-byte reads within a stage
    uint32_t lds_off[2][2];
#pragma unroll
    for (int s = 0; s < 2; ++s) {
        const int row = 8 * warp + 4 * s + c;
#pragma unroll
        for (int h = 0; h < 2; ++h) lds_off[s][h] = smem_addr(ring) + h * kBoxBytes + row * 128 + ((L ^ (row & 7)) << 4);
    }
    const uint16_t* arow[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
        const int m = m0 + 8 * mt + r;
        arow[mt] = (m < p.M) ? p.A + (size_t)m * p.K : nullptr;
    }
    const int lane_kw = 8 * warp + c;

    float acc[MT][4][4], dg[MT][4][4], ones[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
        for (int t = 0; t < 4; ++t)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[mt][t][e] = dg[mt][t][e] = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) ones[mt][e] = 0.f;
    }
    uint2 sp[2] = {make_uint2(0, 0), make_uint2(0, 0)};   // scales of the group summed in dg (slots 0-3, 4-7)
    uint2 zp[2] = {make_uint2(0, 0), make_uint2(0, 0)};   // its zero points
    bool pending = false, aborted = false;
    int cur_tile = -1, cur_group = -1;
    uint4 act[2][MT];
    int cidx = chunk_of(0);
    int t = (int)fdiv((uint32_t)cidx, p.cdiv), kc = cidx - t * p.cpt;
    load_activations<MT>(p, act, arow, kc, lane_kw);

    for (int i = 0; i < nch; ++i) {
        const int slot = i & (kStages - 1);
        const uint32_t ph = (uint32_t)((i / kStages) & 1);
        int kc_next = 0, t_next = 0;
        if (i + 1 < nch) {
            const int cn = chunk_of(i + 1);
            t_next = (int)fdiv((uint32_t)cn, p.cdiv);
            kc_next = cn - t_next * p.cpt;
        }
        const int kw0 = kc * kChunkRows + 8 * warp;         // this warp's rows kw0 .. kw0 + 7 (warp-uniform)
        const bool active = kw0 < p.KW;
        if (t != cur_tile) {
            if (pending) flush_group<MT, HAS_ZP>(acc, dg, ones, sp, zp);
            pending = false;
            if (cur_tile >= 0) finish_tile<MT>(p, red, acc, cur_tile, c_begin, c_end, warp, L, c);
            cur_tile = t;
            cur_group = -1;
        }
        if (active) {
            const int g = (int)fdiv((uint32_t)kw0, p.gdiv);
            if (g != cur_group) {
                if (pending) flush_group<MT, HAS_ZP>(acc, dg, ones, sp, zp);
                pending = false;
                load_group<HAS_ZP>(p, sp, zp, g, t, L);     // consumed at the next flush, a chunk later
                cur_group = g;
            }
        }
        if (!aborted && sflag[0]) aborted = true;
        if (!aborted && !mbar_wait_bounded(&full[slot], ph, kWaitLimitNs)) {
            aborted = true;
            sflag[0] = 1;
            atomicOr(p.err, kErrTimeout);
        }
        uint32_t wd[2][8];
        const uint32_t stage = slot * kStageBytes;
#pragma unroll
        for (int s = 0; s < 2; ++s)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                uint4 v = make_uint4(0, 0, 0, 0);
                if (!aborted && active) v = lds128(lds_off[s][h] + stage);
                wd[s][4 * h + 0] = v.x; wd[s][4 * h + 1] = v.y; wd[s][4 * h + 2] = v.z; wd[s][4 * h + 3] = v.w;
            }
        // activation fragments of both steps: pairs (a[2h], a[2h+4]), (a[2h+1], a[2h+5])
        uint32_t bf[2][MT][2][2];
#pragma unroll
        for (int s = 0; s < 2; ++s)
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                const uint4 a = act[s][mt];
                bf[s][mt][0][0] = prmt(a.x, a.z, 0x5410);
                bf[s][mt][0][1] = prmt(a.x, a.z, 0x7632);
                bf[s][mt][1][0] = prmt(a.y, a.w, 0x5410);
                bf[s][mt][1][1] = prmt(a.y, a.w, 0x7632);
            }
        if (i + 1 < nch) load_activations<MT>(p, act, arow, kc_next, lane_kw);
        if (!aborted && active) {
#pragma unroll
            for (int s = 0; s < 2; ++s) {
                if (kw0 + 4 * s >= p.KW) break;
                if constexpr (HAS_ZP) {
#pragma unroll
                    for (int h = 0; h < 2; ++h)
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt)
                            mma_16816(ones[mt], 0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u,
                                      bf[s][mt][h][0], bf[s][mt][h][1]);
                }
#pragma unroll
                for (int t4 = 0; t4 < 4; ++t4) {
                    uint32_t P0[4], P1[4];
                    unpack_w4_exact<SIGNED>(wd[s][2 * t4], P0);
                    unpack_w4_exact<SIGNED>(wd[s][2 * t4 + 1], P1);
#pragma unroll
                    for (int h = 0; h < 2; ++h)
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt)
                            mma_16816(dg[mt][t4], P0[2 * h], P1[2 * h], P0[2 * h + 1], P1[2 * h + 1],
                                      bf[s][mt][h][0], bf[s][mt][h][1]);
                }
            }
            pending = true;
        }
        // The words of this slot are consumed (the MMAs above read them), so
        // the last warp to get here refills the slot with chunk i + kStages.
        __syncwarp();
        if (lane == 0) {
            if (atomicAdd(&readers[slot], 1) == kWarps - 1) {
                readers[slot] = 0;
                if (i + kStages < nch && !sflag[0]) {
                    const int cf = chunk_of(i + kStages);
                    const int tf = (int)fdiv((uint32_t)cf, p.cdiv);
                    fence_proxy_async_smem();
                    issue_chunk(&tmap, ring, full, slot, tf, cf - tf * p.cpt);
                }
            }
        }
        t = t_next;
        kc = kc_next;
    }
    if (pending) flush_group<MT, HAS_ZP>(acc, dg, ones, sp, zp);
    if (cur_tile >= 0) finish_tile<MT>(p, red, acc, cur_tile, c_begin, c_end, warp, L, c);
    if (reducer) reduce_split_tile<MT>(p, t_last, sflag);
    if (aborted && threadIdx.x == 0) {
        // do not leave the CTA while copies may still be landing
        for (int j = (nch > kStages ? nch - kStages : 0); j < nch; ++j)
            mbar_wait_bounded(&full[j & (kStages - 1)], (uint32_t)((j / kStages) & 1), kWaitLimitNs / 4);
    }
}

template <int MT, bool SIGNED, bool HAS_ZP>
int launch(const CUtensorMap& tmap, const StreamParams& p, int ychunks, bool pdl, cudaStream_t stream) {
    constexpr int MR = 8 * MT;
    const size_t smem = 1024 + kStages * kStageBytes + (size_t)kWarps * kTileN * (MR + 1) * 4 + kStages * 8 +
                        kStages * 4 + 16;
    auto kern = gemv_w4_stream_kernel<MT, SIGNED, HAS_ZP>;
    static SmemLimit limit;     // per instantiation, per device
    const int st = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), (int)smem, &limit);
    if (st != T4B_OK) return st;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.G, ychunks, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t err = cudaLaunchKernelEx(&cfg, kern, tmap, p);
    if (err != cudaSuccess) return record_cuda_error(err);
    return T4B_OK;
}

int launch_any(bool is_signed, const CUtensorMap& tmap, const StreamParams& p, bool pdl, cudaStream_t stream) {
    const int y = 1;
    const bool zp = p.Z != nullptr;
    if (p.M <= 8) {
        if (is_signed) return zp ? launch<1, true, true>(tmap, p, y, pdl, stream) : launch<1, true, false>(tmap, p, y, pdl, stream);
        return zp ? launch<1, false, true>(tmap, p, y, pdl, stream) : launch<1, false, false>(tmap, p, y, pdl, stream);
    }
    if (is_signed) return zp ? launch<2, true, true>(tmap, p, y, pdl, stream) : launch<2, true, false>(tmap, p, y, pdl, stream);
    return zp ? launch<2, false, true>(tmap, p, y, pdl, stream) : launch<2, false, false>(tmap, p, y, pdl, stream);
}

// Shape checks, tensor map and work split of one call.  The caller fills in
// the scratch pointers (part, flags, err) before launching.
int plan_stream(const void* A, const void* W, const void* S, const void* Z, void* C, int M, int N, int K, int group,
                CUtensorMap* tmap_out, StreamParams* out, size_t* flag_words, size_t* part_floats) {
    const int KW = K / 8;
    const int gw = group / 8;
    if ((N % 4) != 0 || !aligned(W, 16) || !aligned(S, 8) || (Z && !aligned(Z, 8))) return T4B_ERR_UNSUPPORTED;
    // a warp's 8 rows of a chunk must lie in one scale group
    if (!(gw % 8 == 0 || gw >= KW)) return T4B_ERR_UNSUPPORTED;
    // one row chunk only: the whole grid (one CTA per SM) must be resident,
    // because a split tile's reducer waits for the other segments' flags
    if (M > 16) return T4B_ERR_UNSUPPORTED;
    if (!make_tmap_u32_2d(tmap_out, W, (uint64_t)KW, (uint64_t)N, kChunkRows, kBoxCols)) return T4B_ERR_UNSUPPORTED;
    const int MR = (M <= 8) ? 8 : 16;
    StreamParams p;
    p.A = static_cast<const uint16_t*>(A);
    p.S = static_cast<const uint16_t*>(S);
    p.Z = static_cast<const uint16_t*>(Z);
    p.C = static_cast<uint16_t*>(C);
    p.part = nullptr;
    p.flags = nullptr;
    p.err = nullptr;
    p.M = M; p.N = N; p.K = K; p.KW = KW;
    p.tiles = (N + kTileN - 1) / kTileN;
    p.cpt = (KW + kChunkRows - 1) / kChunkRows;
    const long long total = (long long)p.tiles * p.cpt;
    if (total > (1ll << 30)) return T4B_ERR_UNSUPPORTED;
    p.total = (int)total;
    p.G = (p.total < sm_count()) ? p.total : sm_count();
    p.gdiv = make_fastdiv((uint32_t)gw);
    p.cdiv = make_fastdiv((uint32_t)p.cpt);
    // most CTAs that can share one tile (cta_of is within one of x * G / total)
    int max_segs = 1;
    for (int t = 0; t < p.tiles; ++t) {
        const long long first = (long long)t * p.cpt, last = first + p.cpt - 1;
        const int n = (int)(last * p.G / p.total) - (int)(first * p.G / p.total) + 3;
        if (n > max_segs) max_segs = n;
    }
    p.max_segs = max_segs;
    *part_floats = (size_t)p.tiles * max_segs * kTileN * MR;
    *flag_words = (size_t)p.tiles * max_segs;
    *out = p;
    return T4B_OK;
}

}  // namespace

int gemv_w4_stream(bool is_signed, const void* A, const void* W, const void* S, const void* Z, void* C, int M, int N,
                   int K, int group, cudaStream_t stream) {
    CUtensorMap tmap;
    StreamParams p;
    size_t flag_words = 0, part_floats = 0;
    int st = plan_stream(A, W, S, Z, C, M, N, K, group, &tmap, &p, &flag_words, &part_floats);
    if (st != T4B_OK) return st;
    Workspace ws;
    st = acquire_workspace(stream, flag_words, part_floats, &ws);
    if (st != T4B_OK) return st;
    p.part = ws.part;
    p.flags = ws.counters;
    p.err = ws.error;
    return launch_any(is_signed, tmap, p, /*pdl=*/true, stream);
}

// ---- allocation-free variant ----------------------------------------------
// Some callers cannot allocate device memory while they run: an inference
// server that reserves all of HBM for its own pool up front and hands it out
// itself, a runtime that forbids allocation once serving has started, or code
// that must not touch the allocator at all.  For them the decode GEMV above
// can run on a fixed scratch array that is part of this library's image on
// every GPU that loads it (kept until the process exits), instead of the
// per-stream workspace the library would otherwise cudaMalloc.
//
// Layout of the array: bytes [0, 256) hold the device error word, then the
// per-segment "published" flags, then (at a 256-byte boundary) the partial
// sums of split tiles.  Each call clears the flags it uses with one
// cudaMemsetAsync; the error word stays set once a bounded wait has given up
// (t4b_device_error reads and clears it), and the partials need no clearing
// (every one is written before it is read).  All calls share the array, so
// two calls that overlap on the GPU (different streams, or concurrent graph
// replays) race.
constexpr size_t kStaticScratchBytes = size_t(4) << 20;   // 4 MiB
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// Device address of g_static_scratch on the current device.  The host-side
// name of the array is only a stand-in; the address has to be looked up once
// per device, with that device current.
int static_scratch_address(unsigned char** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return record_cuda_error(e);
    static std::mutex mu;
    static std::vector<unsigned char*> addr;
    std::lock_guard<std::mutex> lock(mu);
    if ((size_t)dev >= addr.size()) addr.resize(dev + 1, nullptr);
    if (!addr[dev]) {
        void* ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_static_scratch);
        if (e != cudaSuccess) return record_cuda_error(e);
        addr[dev] = static_cast<unsigned char*>(ptr);
    }
    *out = addr[dev];
    return T4B_OK;
}

// Reads (and optionally clears) the allocation-free GEMV's error word on the
// current device; synchronizes `stream`.
int static_scratch_error(cudaStream_t stream, unsigned* out, bool clear) {
    unsigned char* base = nullptr;
    int st = static_scratch_address(&base);
    if (st != T4B_OK) return st;
    cudaError_t e = cudaMemcpyAsync(out, base, sizeof(unsigned), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess && clear) e = cudaMemsetAsync(base, 0, sizeof(unsigned), stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    return e == cudaSuccess ? T4B_OK : record_cuda_error(e);
}

}  // namespace t4b

extern "C" int t4b_fused_w4a16_gemv_noalloc(const void* A, const void* W_packed, const void* scales,
                                            const void* zero_points, void* C, int M, int N, int K, int group_size,
                                            int is_signed, void* stream_) {
    using namespace t4b;
    if (M < 1 || N < 1 || K < 8 || (K % 8) != 0) return T4B_ERR_INVALID_VALUE;
    if (group_size < 8 || (group_size % 8) != 0 || (K % group_size) != 0) return T4B_ERR_INVALID_VALUE;
    if (!A || !W_packed || !scales || !C) return T4B_ERR_NULL_POINTER;
    if (!aligned(A, 16) || !aligned(W_packed, 4) || !aligned(scales, 2) || !aligned(C, 2) ||
        (zero_points && !aligned(zero_points, 2)))
        return T4B_ERR_MISALIGNED;
    const cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    CUtensorMap tmap;
    StreamParams p;
    size_t flag_words = 0, part_floats = 0;
    int st = plan_stream(A, W_packed, scales, zero_points, C, M, N, K, group_size, &tmap, &p, &flag_words,
                         &part_floats);
    if (st != T4B_OK) return st;
    const size_t head = 256 + flag_words * sizeof(unsigned);
    const size_t part_off = (head + 255) & ~size_t(255);
    if (part_off + part_floats * sizeof(float) > kStaticScratchBytes) return T4B_ERR_SCRATCH_LIMIT;
    unsigned char* base = nullptr;
    st = static_scratch_address(&base);
    if (st != T4B_OK) return st;
    cudaError_t e = cudaMemsetAsync(base + 256, 0, head - 256, stream);   // the flags, not the error word
    if (e != cudaSuccess) return record_cuda_error(e);
    p.err = reinterpret_cast<unsigned*>(base);
    p.flags = reinterpret_cast<unsigned*>(base + 256);
    p.part = reinterpret_cast<float*>(base + part_off);
    return launch_any(is_signed != 0, tmap, p, /*pdl=*/false, stream);
}
