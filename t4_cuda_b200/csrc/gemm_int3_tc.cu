// Prefill INT3 GEMM (H17 packing) on the 5th-generation tensor cores:
//
//   C[M, N] = A[M, K] x dequant_s3(W)[K, N],  W int32 [K/10, N] (ten signed
//   3-bit values a word along K), group scales (and zero points) [G, N]
//
// for M > 16, K % 10 == 0, an even group >= 64 and N % 8 == 0 -- the same
// operands as the INT3 GEMV (src/kernels/h17_mega_kernel.h:10-30), which
// keeps M <= 16 and every shape this kernel declines.
//
// The single-CTA pipeline of the INT4 prefill GEMM: one CTA per 128 x 256
// tile of C, tcgen05.mma (M = 128, N = 256, K = 16 per instruction, fp16 in,
// fp32 accumulator in TMEM), K in steps of 64 through a 6-deep ring of
// stages and a 2-deep ring of dequantized B tiles.  Warp roles:
//   warp 0      one thread issues the TMA copies of a stage: the 8 word rows
//               x 256 columns of packed words that hold the step's K range,
//               and the two rows of scales (and zero points) it can touch;
//   warp 1      allocates TMEM; one thread issues the step's four MMAs once
//               the stage's A tile and the dequantized B are in place, and
//               commits them to the barriers that free both slots;
//   warps 2-5   copy the 128 x 64 tile of A with cp.async (below);
//   warps 6-21  dequantize into B (256 x 64 fp16, K-major, 128-byte swizzle),
//               then drain the accumulator from TMEM and store C.
//
// A by cp.async.  K is a multiple of 10, so A's row pitch (2K bytes) is in
// general not a multiple of 16 bytes, which a tensor map needs.  The loader
// warps copy each K step's tile with 8-byte (K % 4 == 0) or 4-byte cp.async,
// zero-filled past M and K, into the 128-byte-swizzled K-major layout a TMA
// copy would produce, keep three K steps of copies in flight per thread
// (cp.async groups), and signal a stage once its copies have landed.
//
// Dequant.  K step kg covers K rows [64 kg, 64 kg + 64): from value
// 64 kg mod 10 of word 64 kg / 10 on, so the stage's 8 word rows from there
// hold it (80 values >= 64 + 9).  A dequant thread takes one column and 32
// consecutive K values, which start at value o = (64 kg + 32 h) mod 10 of a
// word (even, the same for the whole warp) and span 4 words; funnel shifts
// re-cut them into words that start at a value boundary, so every o runs the
// same code.  Each fp16 pair of consecutive K values is then two adjacent
// 3-bit fields of one word (o is even), put under the exponent of 1024 with the top bit
// of each field flipped -- 1028 + q exactly -- so q = (1028 + q) - 1028 and
// the weight is fp16(q s), rounded once (fp16(fp32((q - z) s)) with zero
// points).  A step lies in at most two scale groups (group >= 64); a pair
// takes the group of its K (group boundaries are even, so no pair straddles
// one).
//
// Every wait on an mbarrier is bounded; a timeout sets this file's device
// error word, stops the pipeline, and the CTA still drains its copies and
// frees TMEM before it exits.
#include <algorithm>

#include "common.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"
#include "workspace.h"

namespace t4b {
namespace {

constexpr int kBM = 128, kBN = 256, kBK = 64;
constexpr int kStages = 6;
constexpr int kBStages = 2;
constexpr int kLoadWarps = 4;
constexpr int kDqWarps = 16;
constexpr int kDq0 = 2 + kLoadWarps;                   // first dequant warp
constexpr int kThreads = 32 * (kDq0 + kDqWarps);        // 704
constexpr int kABytes = kBM * kBK * 2;                 // 16 KB
constexpr int kWRows = 8;                              // word rows a stage holds
constexpr int kWBytes = kWRows * kBN * 4;              // 8 KB
constexpr int kSBytes = 2 * kBN * 2;                   // two rows of scales
constexpr int kStageBytes = kABytes + kWBytes + 2 * kSBytes;   // 26 KB
constexpr int kBBytes = kBN * kBK * 2;                 // 32 KB
constexpr int kRingBytes = kStages * kStageBytes + kBStages * kBBytes;
constexpr int kBarriers = 3 * kStages + 2 * kBStages + 1;
constexpr int kInFlight = 3;                           // K steps of A copies in flight per loader thread
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr unsigned kErrTimeout = 1u;
constexpr uint32_t kInstrDesc = tc_idesc_f16(kBM, kBN);
constexpr int kMinSplitSteps = 8;       // K steps a split takes at least
constexpr int kMinSplitK = 8192;        // K from which any under-filled grid splits K
constexpr int kMinPairSplitSteps = 96;  // K steps a split of a CTA pair takes at least
constexpr int kMinLooseSplitSteps = 16; // ... when the grid fills more than a quarter of the SMs
constexpr int kRedPitch = kBN + 1;      // a CTA's fp32 tile in shared memory (cluster split), row pitch
static_assert(kBM * kRedPitch * 4 <= kRingBytes, "a CTA's fp32 tile fits in its ring");
static_assert(kStageBytes % 1024 == 0, "every A tile 1024-byte aligned");
static_assert(kStages > kInFlight, "a stage is signalled before the loader needs its slot again");

// Device error word of this kernel, one per device (int3_tc_device_error).
__device__ unsigned g_int3_tc_error = 0;

struct Int3TcParams {
    const uint16_t* A;
    uint16_t* C;
    int M, N, K;
    int group;
    FastDiv gdiv;           // division by group
    int ksteps;             // ceil(K / 64)
    int ksplit, ks_per;     // split K as in the INT4 GEMM
    int cluster_split;      // single-CTA kernel: the splits of a tile are one cluster (else part / counters)
    float* part;            // [tiles][ksplit][128][256]
    unsigned* counters;     // one per tile, zero between launches
};

struct Int3TcMaps {
    CUtensorMap w;      // W [K/10, N] u32, box 256 x 8
    CUtensorMap s;      // scales [G, N] fp16, box 256 x 2
    CUtensorMap z;      // zero points, same (unused without them)
};

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (mbar_wait_bounded(bar, parity, kWaitLimitNs)) return true;
    *abort_flag = 1;
    atomicOr(&g_int3_tc_error, kErrTimeout);
    return false;
}

__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async8(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// This warp's 32 rows of the 128 x 64 A tile of K step kg, into the stage at
// shared address dst0: row R at R * 128 bytes, 16-byte unit j at
// (j ^ (R & 7)) -- the layout of a 128-byte-swizzled TMA box.
template <bool A8>
__device__ __forceinline__ void copy_a(const Int3TcParams& p, uint32_t dst0, int m0, int row0, int kg, int lane) {
    if constexpr (A8) {
        // lanes 0-15 one row, 16-31 the next: 16 x 8 bytes = the row's 64 K
        const int k = kg * kBK + 4 * (lane & 15);
        const bool kin = k < p.K;             // K % 4 == 0: all 4 values in or all out
#pragma unroll 8
        for (int r = 0; r < 16; ++r) {
            const int R = row0 + 2 * r + (lane >> 4);
            const bool in = kin && (m0 + R < p.M);
            const uint32_t dst = dst0 + (uint32_t)R * 128u + ((uint32_t)(((lane & 15) >> 1) ^ (R & 7)) << 4) +
                                 (uint32_t)(lane & 1) * 8u;
            const uint16_t* src = in ? p.A + (size_t)(m0 + R) * p.K + k : p.A;
            cp_async8(dst, src, in ? 8u : 0u);
        }
    } else {
        // one row per warp instruction, 2 K values a lane
        const int k = kg * kBK + 2 * lane;
        const bool kin = k < p.K;             // K even: both values in or both out
#pragma unroll 8
        for (int r = 0; r < 32; ++r) {
            const int R = row0 + r;
            const bool in = kin && (m0 + R < p.M);
            const uint32_t dst = dst0 + (uint32_t)R * 128u + ((uint32_t)((lane >> 2) ^ (R & 7)) << 4) +
                                 (uint32_t)(lane & 3) * 4u;
            const uint16_t* src = in ? p.A + (size_t)(m0 + R) * p.K + k : p.A;
            cp_async4(dst, src, in ? 4u : 0u);
        }
    }
}

// Fields f and f + 1 (f even) of w as fp16x2 1028 + q (low half field f).
__device__ __forceinline__ uint32_t pair_s3(uint32_t w, int f) {
    const uint32_t lo = w >> (3 * f);
    const uint32_t hi = (f <= 4) ? (w << (13 - 3 * f)) : (w >> (3 * f - 13));   // field f + 1 to bits 16-18
    const uint32_t a = lop3<0x6A>(lo, 0x7u, 0x64046404u);           // (lo & 7) ^ (1024 | 4 in each half)
    return lop3<0x6A>(hi, 0x00070000u, a);
}

// Scales (and zero points) of the two groups a step can touch.
struct PairScales {
    uint32_t s2[2];     // fp16x2 (no zero points)
    float s[2], z[2];   // with zero points
};

// One dequant thread's 32 values of column n, as the four 16-byte units
// j = 4h .. 4h + 3 of B row n.  nw: the values as aligned words -- pair i is
// fields 2 (i % 5), 2 (i % 5) + 1 of nw[i / 5] (bits 30-31 are not read).  Pair i takes the scales of
// group 1 if MIXED and i >= cb, else those of group 0.
template <bool HAS_ZP, bool MIXED>
__device__ __forceinline__ void dequant_vals(const uint32_t (&nw)[4], const PairScales& ps, int cb, uint8_t* brow,
                                             int n, int h) {
    // exact q pairs: words 0-2 whole (unpack_s3_exact gives (e_i, e_{i+5}),
    // five byte permutes make the consecutive pairs), pair 15 from word 3
    uint32_t qp[16];
#pragma unroll
    for (int u = 0; u < 3; ++u) {
        uint32_t p[5];
        unpack_s3_exact(nw[u], p);
        qp[5 * u + 0] = prmt(p[0], p[1], 0x5410u);     // (e0, e1)
        qp[5 * u + 1] = prmt(p[2], p[3], 0x5410u);     // (e2, e3)
        qp[5 * u + 2] = prmt(p[4], p[0], 0x7610u);     // (e4, e5)
        qp[5 * u + 3] = prmt(p[1], p[2], 0x7632u);     // (e6, e7)
        qp[5 * u + 4] = prmt(p[3], p[4], 0x7632u);     // (e8, e9)
    }
    qp[15] = h2_sub(pair_s3(nw[3], 0), H2_1028);
#pragma unroll
    for (int u4 = 0; u4 < 4; ++u4) {
        uint32_t o4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int i = 4 * u4 + e;
            const uint32_t q = qp[i];
            const bool second = MIXED && i >= cb;
            if constexpr (HAS_ZP) {
                const float sf = second ? ps.s[1] : ps.s[0];
                const float zf = second ? ps.z[1] : ps.z[0];
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&q));
                o4[e] = f2_to_h2((f.x - zf) * sf, (f.y - zf) * sf);
            } else {
                o4[e] = h2_mul(q, second ? ps.s2[1] : ps.s2[0]);
            }
        }
        const int j = 4 * h + u4;
        *reinterpret_cast<uint4*>(brow + ((j ^ (n & 7)) << 4)) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
    }
}

// One K step of one dequant thread: column n of a tile of COLS columns, K
// values [k0 + 32 h, k0 + 32 h + 32), which start at field o of a packed word
// (o even) and span 4 words.  They are first re-cut into words that start at
// a value boundary (nw[u] = fields o + 10 u .. o + 10 u + 9 of the stream,
// funnel-shifted from two words, the unused top bits dropped), so one code
// path serves every o.  st_w: the stage's packed words (8 rows x COLS), st_s:
// its two scale rows (and two zero-point rows after them), brow: row n of the
// B slot.  cb >= 16: every pair in group 0; cb <= 0: every pair in group 1
// (moved to index 0); else the step's group boundary falls inside this
// thread's values.
template <int COLS, bool HAS_ZP>
__device__ __forceinline__ void dequant_step(const uint32_t* st_w, const uint16_t* st_s, int k0, int h, int n,
                                             const FastDiv& gdiv, int group, uint8_t* brow) {
    const int klo = k0 + 32 * h;
    const int wq = klo / 10;
    const int o = klo - 10 * wq;                      // 0, 2, 4, 6 or 8 (warp-uniform)
    const uint32_t* wp = st_w + (wq - k0 / 10) * COLS + n;
    uint32_t w[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) w[u] = wp[u * COLS];
    // (w[u + 1] : w[u] << 2) >> (3 o + 2): w[u]'s 30 value bits from field o
    // on, then w[u + 1]'s; bits 30-31 of the result are never read
    const uint32_t sh = 3u * (uint32_t)o;
    uint32_t nw[4];
#pragma unroll
    for (int u = 0; u < 3; ++u) nw[u] = __funnelshift_r(w[u] << 2, w[u + 1], sh + 2u);
    nw[3] = w[3] >> sh;                               // pair 15: fields o, o + 1 of w[3]
    PairScales ps = {};
    const int kb = ((int)fdiv((uint32_t)k0, gdiv) + 1) * group;   // first K of the step's second group
    const int cb = (kb - klo) >> 1;                   // this thread's pairs before it (may be < 0)
    ps.s2[0] = h2_dup(st_s[n]);
    ps.s2[1] = h2_dup(st_s[COLS + n]);
    if constexpr (HAS_ZP) {
        ps.s[0] = h_to_f(st_s[n]);
        ps.s[1] = h_to_f(st_s[COLS + n]);
        ps.z[0] = h_to_f(st_s[2 * COLS + n]);
        ps.z[1] = h_to_f(st_s[3 * COLS + n]);
    }
    if (cb > 0 && cb < 16) {
        dequant_vals<HAS_ZP, true>(nw, ps, cb, brow, n, h);
        return;
    }
    if (cb <= 0) {
        ps.s2[0] = ps.s2[1];
        ps.s[0] = ps.s[1];
        ps.z[0] = ps.z[1];
    }
    dequant_vals<HAS_ZP, false>(nw, ps, cb, brow, n, h);
}

template <bool HAS_ZP, bool A8>
__global__ void __launch_bounds__(kThreads, 1)
gemm_int3_tc_kernel(const __grid_constant__ Int3TcMaps maps, const Int3TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    // stage s: [A 16 KB][packed 8 KB][scales 2 x 512 B][zero points 2 x 512 B]; then the B slots
    uint8_t* bring = base + kStages * kStageBytes;
    uint64_t* full_w = reinterpret_cast<uint64_t*>(base + kRingBytes);   // TMA: words + scales
    uint64_t* full_a = full_w + kStages;                                 // loader warps: A
    uint64_t* empty = full_a + kStages;                                  // tcgen05.commit
    uint64_t* full_b = empty + kStages;
    uint64_t* empty_b = full_b + kBStages;
    uint64_t* acc_full = empty_b + kBStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* last_flag = abort_flag + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_launch_dependents();     // the next kernel may start its prologue as SMs free up
    const int n0 = blockIdx.x * kBN, m0 = blockIdx.y * kBM;
    const int k_begin = blockIdx.z * p.ks_per;
    const int nsteps = min(p.ks_per, p.ksteps - k_begin);     // >= 1: the host sizes the split so

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full_w[s], 1);
            mbar_init(&full_a[s], kLoadWarps);
            mbar_init(&empty[s], 1);
        }
        for (int s = 0; s < kBStages; ++s) {
            mbar_init(&full_b[s], kDqWarps);
            mbar_init(&empty_b[s], 1);
        }
        mbar_init(acc_full, 1);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tmap(&maps.w);
        prefetch_tmap(&maps.s);
        if constexpr (HAS_ZP) prefetch_tmap(&maps.z);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(kBN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_d = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer: packed words and scale rows
        if (lane == 0) {
            // packed words and scales only: never written by a kernel of this
            // library, so no dependency wait (the A loaders wait)
            for (int i = 0; i < nsteps; ++i) {
                const int s = i % kStages;
                if (i >= kStages && !wait_or_abort(&empty[s], (uint32_t)(((i / kStages) & 1) ^ 1), abort_flag)) break;
                uint8_t* st = base + s * kStageBytes;
                const int k0 = (k_begin + i) * kBK;
                const int g0 = (int)fdiv((uint32_t)k0, p.gdiv);
                mbar_arrive_expect_tx(&full_w[s], kWBytes + kSBytes * (HAS_ZP ? 2 : 1));
                tma_load_2d(st + kABytes, &maps.w, n0, k0 / 10, &full_w[s]);
                tma_load_2d(st + kABytes + kWBytes, &maps.s, n0, g0, &full_w[s]);
                if constexpr (HAS_ZP) tma_load_2d(st + kABytes + kWBytes + kSBytes, &maps.z, n0, g0, &full_w[s]);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer
        if (lane == 0) {
            for (int i = 0; i < nsteps; ++i) {
                const int s = i % kStages, b = i % kBStages;
                if (!wait_or_abort(&full_a[s], (uint32_t)((i / kStages) & 1), abort_flag)) break;
                if (!wait_or_abort(&full_b[b], (uint32_t)((i / kBStages) & 1), abort_flag)) break;
                const uint32_t a_addr = smem_addr(base + s * kStageBytes);
                const uint32_t b_addr = smem_addr(bring + b * kBBytes);
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk)
                    tc_mma_f16(tmem_d, smem_desc_sw128(a_addr + kk * 32), smem_desc_sw128(b_addr + kk * 32),
                               kInstrDesc, (i > 0 || kk > 0) ? 1u : 0u);
                tc_commit(&empty[s]);       // both fire once these MMAs have read their operands
                tc_commit(&empty_b[b]);
            }
            tc_commit(acc_full);            // fires once every MMA issued above has completed
        }
    } else if (warp < kDq0) {
        // ---------------- A loaders: cp.async, kInFlight steps of groups in flight
        const int row0 = 32 * (warp - 2);
        pdl_wait_prior_grid();       // A may be the previous kernel's output
        int signalled = 0, issued = 0;
        for (int i = 0; i < nsteps; ++i) {
            const int s = i % kStages;
            bool ok = i < kStages || wait_or_abort(&empty[s], (uint32_t)(((i / kStages) & 1) ^ 1), abort_flag);
            if (!__all_sync(0xffffffffu, ok)) break;
            copy_a<A8>(p, smem_addr(base + s * kStageBytes), m0, row0, k_begin + i, lane);
            cp_async_commit();
            ++issued;
            if (issued - signalled == kInFlight) {
                cp_async_wait<kInFlight - 1>();      // the oldest group has landed
                fence_proxy_async_smem();            // generic-proxy writes before the MMA reads them
                __syncwarp();
                if (lane == 0) mbar_arrive(&full_a[signalled % kStages]);
                ++signalled;
            }
        }
        cp_async_wait<0>();
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0)
            for (; signalled < issued; ++signalled) mbar_arrive(&full_a[signalled % kStages]);
    } else {
        // ---------------- dequant warps, then epilogue
        const int t = threadIdx.x - 32 * kDq0;        // 0 .. 511
        const int n = t & (kBN - 1);                  // column of the tile
        const int h = t >> 8;                         // which 32 of the step's 64 K values
        for (int i = 0; i < nsteps; ++i) {
            const int s = i % kStages, b = i % kBStages;
            if (!wait_or_abort(&full_w[s], (uint32_t)((i / kStages) & 1), abort_flag)) break;
            if (i >= kBStages && !wait_or_abort(&empty_b[b], (uint32_t)(((i / kBStages) & 1) ^ 1), abort_flag)) break;
            const uint8_t* st = base + s * kStageBytes;
            dequant_step<kBN, HAS_ZP>(reinterpret_cast<const uint32_t*>(st + kABytes),
                                      reinterpret_cast<const uint16_t*>(st + kABytes + kWBytes), (k_begin + i) * kBK,
                                      h, n, p.gdiv, p.group, bring + b * kBBytes + n * 128);
            fence_proxy_async_smem();      // generic-proxy writes of B before the MMA reads them
            __syncwarp();
            if (lane == 0) mbar_arrive(&full_b[b]);
        }
        // ---------------- epilogue: TMEM lanes 32 * (warp % 4) .. +31 = rows of the tile
        pdl_wait_prior_grid();       // before any store: the previous kernel may read or write C
        const bool ok = wait_or_abort(acc_full, 0, abort_flag);
        tc_fence_after();
        const int quarter = warp & 3;                       // TMEM lanes this warp may read
        const int cq = (warp - kDq0) >> 2;                  // which 64 columns
        const int r = 32 * quarter + lane;
        if (p.ksplit > 1 && p.cluster_split) {
            // Split K in a cluster: the fp32 tile goes to this CTA's ring (idle
            // once acc_full has fired), rows kRedPitch floats apart; the peers
            // add the tiles after the cluster barrier below.
            if (ok) {
                float* tile = reinterpret_cast<float*>(base);
                for (int c0 = 64 * cq; c0 < 64 * cq + 64; c0 += 32) {
                    uint32_t v[32];
                    tmem_ld32(tmem_d + ((uint32_t)(32 * quarter) << 16) + (uint32_t)c0, v);   // warp-collective
#pragma unroll
                    for (int k = 0; k < 32; ++k) tile[r * kRedPitch + c0 + k] = __uint_as_float(v[k]);
                }
            }
        } else if (p.ksplit > 1) {
            // Split K: the fp32 tile goes to this CTA's partial slot; the last
            // CTA of the tile to arrive sums the partials in split order (the
            // same sum whichever CTA is last).  Every thread reaches both
            // barriers and every CTA counts its arrival, so the counter is
            // back at zero after the launch even after an abort.
            const int tile = blockIdx.y * gridDim.x + blockIdx.x;
            float* mine = p.part + (((size_t)tile * p.ksplit + blockIdx.z) * kBM + r) * kBN;
            if (ok) {
                for (int c0 = 64 * cq; c0 < 64 * cq + 64; c0 += 32) {
                    uint32_t v[32];
                    tmem_ld32(tmem_d + ((uint32_t)(32 * quarter) << 16) + (uint32_t)c0, v);   // warp-collective
                    if (m0 + r < p.M) {
#pragma unroll
                        for (int k = 0; k < 32; k += 4)
                            __stcg(reinterpret_cast<float4*>(mine + c0 + k),
                                   make_float4(__uint_as_float(v[k]), __uint_as_float(v[k + 1]),
                                               __uint_as_float(v[k + 2]), __uint_as_float(v[k + 3])));
                    }
                }
            }
            __threadfence();
            asm volatile("bar.sync 1, %0;" ::"n"(32 * kDqWarps) : "memory");
            if (t == 0) {
                const bool last = atomicAdd(p.counters + tile, 1u) == (unsigned)(p.ksplit - 1);
                if (last) p.counters[tile] = 0u;
                *last_flag = last ? 1 : 0;
                __threadfence();
            }
            asm volatile("bar.sync 1, %0;" ::"n"(32 * kDqWarps) : "memory");
            if (ok && *last_flag != 0) {
                constexpr int kPer = kBM * kBN / 4;                  // float4s in a partial
                const int valid = min(kBM, p.M - m0) * (kBN / 4);    // float4s of the tile's rows < M
                const float4* src = reinterpret_cast<const float4*>(p.part) + (size_t)tile * p.ksplit * kPer;
                for (int idx = t; idx < valid; idx += 32 * kDqWarps) {
                    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                    for (int z0 = 0; z0 < p.ksplit; z0 += 4) {
                        float4 f[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u)
                            f[u] = (z0 + u < p.ksplit) ? __ldcg(src + (size_t)(z0 + u) * kPer + idx)
                                                       : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            acc.x += f[u].x; acc.y += f[u].y; acc.z += f[u].z; acc.w += f[u].w;
                        }
                    }
                    const int gr = m0 + (idx >> 6), gc = n0 + ((idx & 63) << 2);
                    if (gr < p.M && gc < p.N) {       // N % 8 == 0: a float4 is all in or all out
                        uint2 o;
                        o.x = f2_to_h2(acc.x, acc.y);
                        o.y = f2_to_h2(acc.z, acc.w);
                        *reinterpret_cast<uint2*>(p.C + (size_t)gr * p.N + gc) = o;
                    }
                }
            }
        } else if (ok) {
            const int row = m0 + r;
            for (int c0 = 64 * cq; c0 < 64 * cq + 64; c0 += 32) {
                uint32_t v[32];
                tmem_ld32(tmem_d + ((uint32_t)(32 * quarter) << 16) + (uint32_t)c0, v);
                if (row < p.M && n0 + c0 < p.N) {
                    uint16_t* crow = p.C + (size_t)row * p.N + n0 + c0;
                    if (n0 + c0 + 32 <= p.N) {
#pragma unroll
                        for (int k = 0; k < 32; k += 8) {
                            uint4 o;
                            o.x = f2_to_h2(__uint_as_float(v[k + 0]), __uint_as_float(v[k + 1]));
                            o.y = f2_to_h2(__uint_as_float(v[k + 2]), __uint_as_float(v[k + 3]));
                            o.z = f2_to_h2(__uint_as_float(v[k + 4]), __uint_as_float(v[k + 5]));
                            o.w = f2_to_h2(__uint_as_float(v[k + 6]), __uint_as_float(v[k + 7]));
                            *reinterpret_cast<uint4*>(crow + k) = o;
                        }
                    } else {
#pragma unroll
                        for (int k = 0; k < 32; ++k)
                            if (n0 + c0 + k < p.N) crow[k] = __half_as_ushort(__float2half_rn(__uint_as_float(v[k])));
                    }
                }
            }
        }
    }

    if (p.ksplit > 1 && p.cluster_split) {
        // Every thread of every CTA of the cluster (one tile, its K splits)
        // passes both barriers, whatever path it took above.
        cluster_sync_all();      // every CTA's fp32 tile is in its shared memory
        if (warp >= kDq0 && !*abort_flag) {
            // CTA `rank` adds its share of the tile's elements (rows < M) over
            // the splits in split order and stores C
            const int ks = p.ksplit;
            const int rank = (int)cluster_rank();
            const int rows = min(kBM, p.M - m0);
            const int E = rows * kBN;
            const int per = (E + ks - 1) / ks;
            const int e_end = min(E, (rank + 1) * per);
            uint32_t peer[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) peer[q] = map_to_rank(base, (uint32_t)(q < ks ? q : 0));
            for (int e = rank * per + (int)threadIdx.x - 32 * kDq0; e < e_end; e += 32 * kDqWarps) {
                const int rr = e >> 8, c = e & (kBN - 1);
                const uint32_t off = (uint32_t)(rr * kRedPitch + c) * 4u;
                float v = 0.f;
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    if (q < ks) v += ld_dsmem_f32(peer[q] + off);
                if (n0 + c < p.N) p.C[(size_t)(m0 + rr) * p.N + n0 + c] = __half_as_ushort(__float2half_rn(v));
            }
        }
        cluster_sync_all();      // no CTA leaves while a peer still reads its tile
    }

    // ---------------- teardown: no MMA may still be writing TMEM when it is freed
    tc_fence_before();
    __syncthreads();
    if (*abort_flag && threadIdx.x == 32) {
        mbar_wait_bounded(acc_full, 0, kWaitLimitNs / 4);
        for (int s = 0; s < kStages; ++s) mbar_wait_bounded(&full_w[s], 0, kWaitLimitNs / 8);
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(kBN));
    }
}

// =============================================================================
// CTA-pair form (M > 128): a cluster of two CTAs runs tcgen05.mma.cta_group::2
// (M = 256, N = 256) on a 256 x 256 tile of C.  Each CTA copies its own 128
// rows of A and dequantizes 128 of the pair's 256 weight columns into its half
// of B, so an SM dequantizes half the columns per MMA tile of the single-CTA
// kernel -- the dequant is what bounds that kernel.  Warp roles per CTA:
//   warp 0      TMA: this CTA's 8 word rows x 128 columns and scale rows;
//   warp 1      allocates the pair's TMEM; in the leader one thread issues a
//               stage's MMAs once both CTAs' A copies (full_a) and B halves
//               (full_b) are in, and commits them to "done" in both CTAs;
//   warps 2-5   cp.async of this CTA's A rows; they arrive on the leader's
//               full_a (a cluster-scope remote arrive from the other CTA);
//   warps 6-13  dequantize, arrive on the leader's full_b, and drain this
//               CTA's 128 accumulator rows.
// "done[s]" frees stage slot s (TMA and A) and B slot (i - kBStages) % kBStages.
// No copy writes or signals the other CTA's shared memory, and no load is a
// multicast.
namespace pair {

constexpr int kRows = 128;                          // rows of A per CTA
constexpr int kCols = 256;                          // columns of C per pair
constexpr int kHalf = 128;                          // B columns per CTA
constexpr int kStages = 6;
constexpr int kBStages = 4;
constexpr int kDqWarps = 8;
constexpr int kThreads = 32 * (kDq0 + kDqWarps);     // 448
constexpr int kWBytes = kWRows * kHalf * 4;          // 4 KB
constexpr int kSBytes = 2 * kHalf * 2;               // two rows of scales
constexpr int kStageBytes = kABytes + kWBytes + 2 * kSBytes;   // 21 KB
constexpr int kBBytes = kHalf * kBK * 2;             // 16 KB
constexpr int kRingBytes = kStages * kStageBytes + kBStages * kBBytes;
constexpr int kBarriers = 3 * kStages + kBStages + 1;
constexpr uint32_t kInstrDesc = tc_idesc_f16(2 * kRows, kCols);
static_assert(kStageBytes % 1024 == 0 && kBBytes % 1024 == 0, "1024-byte aligned operand tiles");
static_assert(kStages > kInFlight && kStages > kBStages, "slot reuse");

__device__ __forceinline__ bool wait_pair(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    return wait_or_abort(bar, parity, abort_flag);
}

template <bool HAS_ZP, bool A8>
__global__ void __launch_bounds__(kThreads, 1)
gemm_int3_tc_pair_kernel(const __grid_constant__ Int3TcMaps maps, const Int3TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    // the same offsets in both CTAs: the MMA addresses the partner's operands
    // by this CTA's shared-memory offsets
    uint8_t* base = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    uint8_t* bring = base + kStages * kStageBytes;
    uint64_t* full_w = reinterpret_cast<uint64_t*>(base + kRingBytes);   // own TMA
    uint64_t* full_a = full_w + kStages;             // leader only: both CTAs' loader warps
    uint64_t* done = full_a + kStages;               // both: the leader's commits
    uint64_t* full_b = done + kStages;               // leader only: both CTAs' dequant warps
    uint64_t* acc_full = full_b + kBStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* last_flag = abort_flag + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_launch_dependents();     // the next kernel may start its prologue as SMs free up
    const uint32_t rank = cluster_rank();            // 0 = leader (issues the MMAs)
    const int pair_id = blockIdx.x >> 1;             // clusters of 2 along x, column tiles fastest
    const int n_tiles = (p.N + kCols - 1) / kCols;
    const int n0 = (pair_id % n_tiles) * kCols;
    const int nh = n0 + (int)rank * kHalf;           // this CTA's B columns
    const int m0 = (pair_id / n_tiles) * (2 * kRows) + (int)rank * kRows;   // this CTA's rows
    const int k_begin = blockIdx.y * p.ks_per;
    const int nsteps = min(p.ks_per, p.ksteps - k_begin);   // >= 1: the host sizes the split so

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full_w[s], 1);
            mbar_init(&full_a[s], 2 * kLoadWarps);
            mbar_init(&done[s], 1);
        }
        for (int b = 0; b < kBStages; ++b) mbar_init(&full_b[b], 2 * kDqWarps);
        mbar_init(acc_full, 1);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tmap(&maps.w);
        prefetch_tmap(&maps.s);
        if constexpr (HAS_ZP) prefetch_tmap(&maps.z);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(kCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    tc_fence_before();
    cluster_sync_all();          // both CTAs' barriers initialised before any remote arrive or commit
    tc_fence_after();
    const uint32_t tmem_d = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer: this CTA's packed words and scale rows
        if (lane == 0) {
            // packed words and scales only: never written by a kernel of this
            // library, so no dependency wait (the A loaders wait)
            for (int i = 0; i < nsteps; ++i) {
                const int s = i % kStages;
                if (i >= kStages && !wait_pair(&done[s], (uint32_t)(((i / kStages) & 1) ^ 1), abort_flag)) break;
                uint8_t* st = base + s * kStageBytes;
                const int k0 = (k_begin + i) * kBK;
                const int g0 = (int)fdiv((uint32_t)k0, p.gdiv);
                mbar_arrive_expect_tx(&full_w[s], kWBytes + kSBytes * (HAS_ZP ? 2 : 1));
                tma_load_2d(st + kABytes, &maps.w, nh, k0 / 10, &full_w[s]);
                tma_load_2d(st + kABytes + kWBytes, &maps.s, nh, g0, &full_w[s]);
                if constexpr (HAS_ZP) tma_load_2d(st + kABytes + kWBytes + kSBytes, &maps.z, nh, g0, &full_w[s]);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (leader CTA only)
        if (rank == 0 && lane == 0) {
            const uint32_t done0 = map_to_rank(&done[0], 0), done1 = map_to_rank(&done[0], 1);
            for (int i = 0; i < nsteps; ++i) {
                const int s = i % kStages, b = i % kBStages;
                if (!wait_pair(&full_a[s], (uint32_t)((i / kStages) & 1), abort_flag)) break;
                if (!wait_pair(&full_b[b], (uint32_t)((i / kBStages) & 1), abort_flag)) break;
                const uint32_t a_addr = smem_addr(base + s * kStageBytes);
                const uint32_t b_addr = smem_addr(bring + b * kBBytes);
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk)
                    tc_mma_pair_f16(tmem_d, smem_desc_sw128(a_addr + kk * 32), smem_desc_sw128(b_addr + kk * 32),
                                    kInstrDesc, (i > 0 || kk > 0) ? 1u : 0u);
                commit_pair(done0 + (uint32_t)(s * 8));     // fire once these MMAs have read their operands
                commit_pair(done1 + (uint32_t)(s * 8));
            }
            commit_pair(map_to_rank(acc_full, 0));     // fire once every MMA issued above has completed
            commit_pair(map_to_rank(acc_full, 1));
        }
    } else if (warp < kDq0) {
        // ---------------- A loaders: this CTA's rows, kInFlight steps of groups in flight
        const int row0 = 32 * (warp - 2);
        pdl_wait_prior_grid();       // A may be the previous kernel's output
        const uint32_t full_a_leader = map_to_rank(&full_a[0], 0);
        int signalled = 0, issued = 0;
        for (int i = 0; i < nsteps; ++i) {
            const int s = i % kStages;
            bool ok = i < kStages || wait_pair(&done[s], (uint32_t)(((i / kStages) & 1) ^ 1), abort_flag);
            if (!__all_sync(0xffffffffu, ok)) break;
            copy_a<A8>(p, smem_addr(base + s * kStageBytes), m0, row0, k_begin + i, lane);
            cp_async_commit();
            ++issued;
            if (issued - signalled == kInFlight) {
                cp_async_wait<kInFlight - 1>();      // the oldest group has landed
                fence_proxy_async_smem();            // generic-proxy writes before the MMA reads them
                __syncwarp();
                if (lane == 0) arrive_cluster(full_a_leader + (uint32_t)((signalled % kStages) * 8));
                ++signalled;
            }
        }
        cp_async_wait<0>();
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0)
            for (; signalled < issued; ++signalled) arrive_cluster(full_a_leader + (uint32_t)((signalled % kStages) * 8));
    } else {
        // ---------------- dequant warps, then epilogue
        const int t = threadIdx.x - 32 * kDq0;        // 0 .. 255
        const int n = t & (kHalf - 1);                // column of this CTA's half
        const int h = t / kHalf;                      // which 32 of the step's 64 K values
        const uint32_t full_b_leader = map_to_rank(&full_b[0], 0);
        for (int i = 0; i < nsteps; ++i) {
            const int s = i % kStages, b = i % kBStages;
            if (!wait_pair(&full_w[s], (uint32_t)((i / kStages) & 1), abort_flag)) break;
            if (i >= kBStages) {
                const int r = i - kBStages;
                if (!wait_pair(&done[r % kStages], (uint32_t)((r / kStages) & 1), abort_flag)) break;
            }
            const uint8_t* st = base + s * kStageBytes;
            dequant_step<kHalf, HAS_ZP>(reinterpret_cast<const uint32_t*>(st + kABytes),
                                        reinterpret_cast<const uint16_t*>(st + kABytes + kWBytes), (k_begin + i) * kBK,
                                        h, n, p.gdiv, p.group, bring + b * kBBytes + n * 128);
            fence_proxy_async_smem();      // generic-proxy writes of B before the MMA reads them
            __syncwarp();
            if (lane == 0) arrive_cluster(full_b_leader + (uint32_t)(b * 8));
        }
        // ---------------- epilogue: TMEM lanes 32 * (warp % 4) .. +31 = this CTA's rows
        pdl_wait_prior_grid();       // before any store: the previous kernel may read or write C
        const bool ok = wait_pair(acc_full, 0, abort_flag);
        tc_fence_after();
        const int quarter = warp & 3;
        constexpr int kColsPerWarp = kCols / (kDqWarps / 4);
        const int cq = (warp - kDq0) >> 2;
        const int r = 32 * quarter + lane;
        if (p.ksplit > 1) {
            // Split K per CTA, as in the single-CTA kernel: this CTA's 128 rows
            // x 256 columns go to their partial slot; the last of the ksplit
            // CTAs holding these rows sums the partials in split order.
            const int tile = 2 * pair_id + (int)rank;
            float* mine = p.part + (((size_t)tile * p.ksplit + blockIdx.y) * kRows + r) * kCols;
            if (ok) {
                for (int c0 = kColsPerWarp * cq; c0 < kColsPerWarp * cq + kColsPerWarp; c0 += 32) {
                    uint32_t v[32];
                    tmem_ld32(tmem_d + ((uint32_t)(32 * quarter) << 16) + (uint32_t)c0, v);   // warp-collective
                    if (m0 + r < p.M) {
#pragma unroll
                        for (int k = 0; k < 32; k += 4)
                            __stcg(reinterpret_cast<float4*>(mine + c0 + k),
                                   make_float4(__uint_as_float(v[k]), __uint_as_float(v[k + 1]),
                                               __uint_as_float(v[k + 2]), __uint_as_float(v[k + 3])));
                    }
                }
            }
            __threadfence();
            asm volatile("bar.sync 1, %0;" ::"n"(32 * kDqWarps) : "memory");
            if (t == 0) {
                const bool last = atomicAdd(p.counters + tile, 1u) == (unsigned)(p.ksplit - 1);
                if (last) p.counters[tile] = 0u;
                *last_flag = last ? 1 : 0;
                __threadfence();
            }
            asm volatile("bar.sync 1, %0;" ::"n"(32 * kDqWarps) : "memory");
            if (ok && *last_flag != 0) {
                constexpr int kPer = kRows * kCols / 4;             // float4s in a partial
                constexpr int kRow4 = kCols / 4;
                const int valid = max(0, min(kRows, p.M - m0)) * kRow4;   // float4s of this CTA's rows < M
                const float4* src = reinterpret_cast<const float4*>(p.part) + (size_t)tile * p.ksplit * kPer;
                for (int idx = t; idx < valid; idx += 32 * kDqWarps) {
                    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                    for (int z0 = 0; z0 < p.ksplit; z0 += 4) {
                        float4 f[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u)
                            f[u] = (z0 + u < p.ksplit) ? __ldcg(src + (size_t)(z0 + u) * kPer + idx)
                                                       : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            acc.x += f[u].x; acc.y += f[u].y; acc.z += f[u].z; acc.w += f[u].w;
                        }
                    }
                    const int gr = m0 + idx / kRow4, gc = n0 + (idx % kRow4) * 4;
                    if (gr < p.M && gc < p.N) {       // N % 8 == 0: a float4 is all in or all out
                        uint2 o;
                        o.x = f2_to_h2(acc.x, acc.y);
                        o.y = f2_to_h2(acc.z, acc.w);
                        *reinterpret_cast<uint2*>(p.C + (size_t)gr * p.N + gc) = o;
                    }
                }
            }
        } else if (ok) {
            const int row = m0 + r;
            for (int c0 = kColsPerWarp * cq; c0 < kColsPerWarp * cq + kColsPerWarp; c0 += 32) {
                uint32_t v[32];
                tmem_ld32(tmem_d + ((uint32_t)(32 * quarter) << 16) + (uint32_t)c0, v);
                if (row < p.M && n0 + c0 < p.N) {
                    uint16_t* crow = p.C + (size_t)row * p.N + n0 + c0;
                    if (n0 + c0 + 32 <= p.N) {
#pragma unroll
                        for (int k = 0; k < 32; k += 8) {
                            uint4 o;
                            o.x = f2_to_h2(__uint_as_float(v[k + 0]), __uint_as_float(v[k + 1]));
                            o.y = f2_to_h2(__uint_as_float(v[k + 2]), __uint_as_float(v[k + 3]));
                            o.z = f2_to_h2(__uint_as_float(v[k + 4]), __uint_as_float(v[k + 5]));
                            o.w = f2_to_h2(__uint_as_float(v[k + 6]), __uint_as_float(v[k + 7]));
                            *reinterpret_cast<uint4*>(crow + k) = o;
                        }
                    } else {
#pragma unroll
                        for (int k = 0; k < 32; ++k)
                            if (n0 + c0 + k < p.N) crow[k] = __half_as_ushort(__float2half_rn(__uint_as_float(v[k])));
                    }
                }
            }
        }
    }

    // ---------------- teardown
    tc_fence_before();
    __syncthreads();
    if (*abort_flag && threadIdx.x == 32) {
        mbar_wait_bounded(acc_full, 0, kWaitLimitNs / 4);
        for (int s = 0; s < kStages; ++s) mbar_wait_bounded(&full_w[s], 0, kWaitLimitNs / 8);
    }
    __syncthreads();
    cluster_sync_all();          // neither CTA frees TMEM or exits while the other may still signal it
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(kCols));
    }
}

template <bool HAS_ZP, bool A8>
int launch(const Int3TcMaps& maps, const Int3TcParams& p, cudaStream_t stream) {
    auto kern = gemm_int3_tc_pair_kernel<HAS_ZP, A8>;
    const size_t smem = 1024 + (size_t)kRingBytes + kBarriers * 8 + 16;
    static SmemLimit limit;     // per instantiation, per device
    const int st = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), (int)smem, &limit);
    if (st != T4B_OK) return st;
    cudaLaunchConfig_t cfg = {};
    const int pairs = ((p.N + kCols - 1) / kCols) * ((p.M + 2 * kRows - 1) / (2 * kRows));
    cfg.gridDim = dim3(2 * pairs, p.ksplit, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;      // the two CTAs of an MMA pair are adjacent along x
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;   // as in the single-CTA launch
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, maps, p);
    if (e != cudaSuccess) return record_cuda_error(e);
    return check_launch();
}

}  // namespace pair

template <bool HAS_ZP, bool A8>
int launch(const Int3TcMaps& maps, const Int3TcParams& p, cudaStream_t stream) {
    auto kern = gemm_int3_tc_kernel<HAS_ZP, A8>;
    const size_t smem = 1024 + (size_t)kRingBytes + kBarriers * 8 + 16;
    static SmemLimit limit;     // per instantiation, per device
    const int st = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), (int)smem, &limit);
    if (st != T4B_OK) return st;
    dim3 grid((p.N + kBN - 1) / kBN, (p.M + kBM - 1) / kBM, p.ksplit);
    // programmatic dependent launch: the prologue overlaps the previous
    // kernel's tail (the kernel waits for it before reading A or storing);
    // the K splits of a tile form one cluster
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = (unsigned)p.ksplit;
    cfg.attrs = attr;
    cfg.numAttrs = (p.ksplit > 1 && p.cluster_split) ? 2 : 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, maps, p);
    if (e != cudaSuccess) return record_cuda_error(e);
    return check_launch();
}

}  // namespace

namespace {

// Clusters of `ks` single-CTA INT3 GEMM CTAs resident at once, and the largest
// split of `tiles` tiles (at most `ks`) whose clusters all are (1: none).
int cluster_split_of(int tiles, int ks) {
    static ClusterCapacityCache cache;
    const int smem = 1024 + kRingBytes + kBarriers * 8 + 16;
    for (; ks >= 2; --ks)
        if (tiles <= max_active_clusters(reinterpret_cast<const void*>(gemm_int3_tc_kernel<false, true>), smem,
                                         kThreads, ks, &cache))
            return ks;
    return 1;
}

}  // namespace

int int3_tc_device_error(cudaStream_t stream, unsigned* out, bool clear) {
    unsigned* word = nullptr;
    cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&word), g_int3_tc_error);
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, word, sizeof(unsigned), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess && clear) e = cudaMemsetAsync(word, 0, sizeof(unsigned), stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    return e == cudaSuccess ? T4B_OK : record_cuda_error(e);
}

int gemm_int3_tc(const void* A, const void* W, const void* S, const void* Z, void* C, int M, int N, int K, int group,
                 bool any_m, cudaStream_t stream) {
    if (M < 1 || (M <= 16 && !any_m) || K < 10 || (K % 10) != 0 || group < kBK || (group & 1) != 0 || (N % 8) != 0)
        return T4B_ERR_UNSUPPORTED;
    if (!aligned(A, 16) || !aligned(W, 16) || !aligned(S, 16) || (Z && !aligned(Z, 16)) || !aligned(C, 16))
        return T4B_ERR_UNSUPPORTED;
    Int3TcParams p;
    p.A = static_cast<const uint16_t*>(A);
    p.C = static_cast<uint16_t*>(C);
    p.M = M; p.N = N; p.K = K;
    p.group = group;
    p.gdiv = make_fastdiv((uint32_t)group);
    p.ksteps = (K + kBK - 1) / kBK;
    p.ksplit = 1;
    p.ks_per = p.ksteps;
    p.cluster_split = 0;
    p.part = nullptr;
    p.counters = nullptr;
    // M > 128: CTA pairs.  Split K where the tiles (or pairs) leave SMs idle,
    // by the INT4 GEMM's rules (measured there): K >= 8192 or a grid of at
    // most a quarter of the SMs from 8 K steps a split, at most half the SMs
    // from 16; pairs when each split keeps >= 96 K steps, else single CTAs,
    // whose splits add up in a cluster.
    bool use_pair = M > kBM;
    const int sms = sm_count();
    const int tiles = ((M + kBM - 1) / kBM) * ((N + kBN - 1) / kBN);
    const int pair_ctas = 2 * ((M + 2 * kBM - 1) / (2 * kBM)) * ((N + kBN - 1) / kBN);
    const bool long_k = K >= kMinSplitK;
    const bool quarter = 4 * tiles <= sms;
    if (M <= 16) {
        // a decode batch fills one 128-row tile: the dequant of B, which every
        // split shares evenly, is the whole cost, so K splits from 4 K steps a
        // split up to about one CTA per SM (as the FP8 GEMM does)
        const int ks = cluster_split_of(tiles, std::min(std::min(sms / tiles, p.ksteps / 4), 8));
        if (ks >= 2) {
            p.ks_per = (p.ksteps + ks - 1) / ks;
            p.ksplit = (p.ksteps + p.ks_per - 1) / p.ks_per;
            p.cluster_split = 1;
        }
    } else if ((long_k || 2 * tiles <= sms) && tiles < sms && (!use_pair || pair_ctas < sms)) {
        const int min_steps = (long_k || quarter) ? kMinSplitSteps : kMinLooseSplitSteps;
        auto split_of = [&](int ctas) { return std::min(std::min(sms / ctas, p.ksteps / min_steps), 8); };
        if (use_pair) {
            const int kp = (long_k || quarter) ? split_of(pair_ctas) : 1;
            const bool pair_split = kp >= 2 && (p.ksteps + kp - 1) / kp >= kMinPairSplitSteps;
            if (!pair_split && cluster_split_of(tiles, split_of(tiles)) >= 2) use_pair = false;
        }
        const int ctas = use_pair ? pair_ctas : tiles;
        const int ks = use_pair ? split_of(ctas) : cluster_split_of(tiles, split_of(tiles));
        if (ks >= 2 && !use_pair) {
            // single CTAs: the splits of a tile are one cluster (no workspace)
            p.ks_per = (p.ksteps + ks - 1) / ks;
            p.ksplit = (p.ksteps + p.ks_per - 1) / p.ks_per;      // no empty split
            p.cluster_split = 1;
        } else if (ks >= 2) {
            p.ks_per = (p.ksteps + ks - 1) / ks;
            p.ksplit = (p.ksteps + p.ks_per - 1) / p.ks_per;      // no empty split
            Workspace ws;
            const int st = acquire_workspace(stream, (size_t)ctas, (size_t)ctas * p.ksplit * kBM * kBN, &ws);
            if (st != T4B_OK) return st;
            p.part = ws.part;
            p.counters = ws.counters;
        }
    }
    const int G = (K + group - 1) / group;
    const uint32_t wbox = use_pair ? pair::kHalf : kBN;
    Int3TcMaps maps;
    if (!make_tmap_2d_ex(&maps.w, false, W, (uint64_t)(K / 10), (uint64_t)N, kWRows, wbox, 0, 256) ||
        !make_tmap_2d_ex(&maps.s, true, S, (uint64_t)G, (uint64_t)N, 2, wbox, 0, 0))
        return T4B_ERR_UNSUPPORTED;
    if (Z) {
        if (!make_tmap_2d_ex(&maps.z, true, Z, (uint64_t)G, (uint64_t)N, 2, wbox, 0, 0)) return T4B_ERR_UNSUPPORTED;
    } else {
        maps.z = maps.s;
    }
    const bool a8 = (K % 4) == 0;
    if (use_pair) {
        if (Z) return a8 ? pair::launch<true, true>(maps, p, stream) : pair::launch<true, false>(maps, p, stream);
        return a8 ? pair::launch<false, true>(maps, p, stream) : pair::launch<false, false>(maps, p, stream);
    }
    if (Z) return a8 ? launch<true, true>(maps, p, stream) : launch<true, false>(maps, p, stream);
    return a8 ? launch<false, true>(maps, p, stream) : launch<false, false>(maps, p, stream);
}

}  // namespace t4b
