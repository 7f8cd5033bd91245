// Prefill W4A16 GEMM on the 5th-generation tensor cores (tcgen05, TMEM):
//
//   C[M, N] = A[M, K] x dequant(W)[K, N],  W int32 [K/8, N], group scales [K/g, N]
//
// for M > 16, K % 64 == 0 and g % 64 == 0.
//
// One CTA computes a 128 x 256 tile of C with a single-CTA tcgen05.mma
// (M = 128, N = 256, K = 16 per instruction, fp16 in, fp32 accumulate in
// TMEM, 256 TMEM columns), looping over K in steps of 64.  Two shared-memory
// rings: a 5-deep one of TMA copies (A, packed words, scales), deep enough to
// cover the copy latency, and a 2-deep one of dequantized B tiles between the
// dequant warps and the MMA.  Warp roles:
//   warp 0      one thread issues the TMA copies of a stage: the 128 x 64 tile
//               of A (128-byte swizzle, the UMMA K-major canonical layout), the
//               8 x 256 tile of packed words, one row of scales (and zero
//               points) -- each K step lies inside one scale group;
//   warp 1      allocates TMEM; one thread issues the MMAs of a stage once A
//               and the dequantized B are in place and commits them to the
//               "empty" barriers of both slots it read, which frees them;
//   warps 2-17  four warpgroups dequantize the packed tile into B (256 x 64
//               fp16, K-major, 128-byte swizzle; a thread does one column and
//               half the K step) -- the weight rounded exactly as the contract
//               says, fp16(q * s) (fp16(fp32((q - z) * s)) with zero points) --
//               and, after the last K step, drain the accumulator from TMEM
//               (each warpgroup 64 of the 256 columns), convert it to fp16 and
//               store C.  Sixteen warps, because a warpgroup's dequant is
//               latency-bound: with fewer the tensor pipe idles waiting for B.
// Every wait on an mbarrier is bounded; a timeout sets this file's device
// error word, stops the pipeline and still frees TMEM before the CTA exits.
#include <atomic>

#include "common.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"
#include "workspace.h"

namespace t4b {
namespace {

constexpr int kBM = 128, kBN = 256, kBK = 64;
constexpr int kTmaStages = 5;
constexpr int kBStages = 2;
constexpr int kDqWarps = 16;                        // dequant / epilogue warps (four warpgroups)
constexpr int kThreads = 64 + 32 * kDqWarps;         // + TMA warp + MMA warp
constexpr int kABytes = kBM * kBK * 2;              // 16 KB
constexpr int kWBytes = (kBK / 8) * kBN * 4;        // 8 KB packed
constexpr int kSBytes = kBN * 2;                    // one row of scales
constexpr int kBBytes = kBN * kBK * 2;              // 32 KB dequantized
constexpr int kTmaStageBytes = kABytes + kWBytes + 2 * kSBytes;   // A, packed, scales, zero points (25 KB)
constexpr int kRingBytes = kTmaStages * kTmaStageBytes + kBStages * kBBytes;
constexpr int kBarriers = 2 * kTmaStages + 2 * kBStages + 1;
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr unsigned kErrTimeout = 1u;

// Device error word of this kernel, one per device (see gemm_tc_device_error).
__device__ unsigned g_gemm_tc_error = 0;

struct GemmParams {
    uint16_t* C;
    int M, N, K;
    int gw_steps;       // K steps (of 64) per scale group (0: a single group, per-column scales)
    int ksteps;
    // split K (single-CTA kernel): blockIdx.z takes K steps [z * ks_per, ...);
    // each CTA stores its fp32 tile to part, and the last of a tile's CTAs
    // (counter) sums the ksplit partials in split order and writes C
    int ksplit, ks_per;
    // single-CTA kernel: 1 = the ksplit CTAs of a tile are one thread-block
    // cluster and add their fp32 tiles through distributed shared memory; 0 =
    // through global memory (part, counters)
    int cluster_split;
    float* part;            // [tiles][ksplit][128][256]
    unsigned* counters;     // one per tile, zero between launches
};

constexpr int kMinSplitSteps = 8;       // K steps (512 K) a split takes at least
constexpr int kMinSplitK = 8192;        // K below which the GEMM never splits K
constexpr int kMinPairSplitSteps = 96;  // K steps a split of a CTA pair takes at least
constexpr int kMinLooseSplitSteps = 16; // ... when the grid fills more than a quarter of the SMs

struct GemmMaps {
    CUtensorMap a;      // A [M, K] fp16, box 64 x 128, 128-byte swizzle
    CUtensorMap w;      // W [K/8, N] u32, box 256 x 8
    CUtensorMap s;      // scales [K/g, N] fp16, box 256 x 1
    CUtensorMap z;      // zero points, same (unused without them)
};

// ---- tcgen05 (the shared helpers are in tcgen05.cuh)
constexpr uint32_t kInstrDesc = tc_idesc_f16(kBM, kBN);

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
    tc_mma_f16(tmem_d, da, db, kInstrDesc, accumulate);
}

// Bounded wait; on timeout records the error and raises the CTA's abort flag.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (mbar_wait_bounded(bar, parity, kWaitLimitNs)) return true;
    *abort_flag = 1;
    atomicOr(&g_gemm_tc_error, kErrTimeout);
    return false;
}

// Eight consecutive K values (one packed word) of one column as four fp16x2
// in natural order, each the exact integer q (signed or unsigned nibble).
template <bool SIGNED>
__device__ __forceinline__ void unpack_natural(uint32_t w, uint32_t (&q)[4]) {
    // byte i of w holds (q_{2i}, q_{2i+1}) in its low / high nibble; copy it to
    // bytes 0 and 2, then take the low nibble under exponent 2^10 (1024 + n)
    // and the high nibble of byte 2 under exponent 2^6 (64 + n).
    constexpr uint32_t kMask = 0x00F0000Fu;
    constexpr uint32_t kMagic = SIGNED ? 0x54806408u : 0x54006400u;   // signed: top bit of each nibble flipped
    constexpr uint32_t kBias = SIGNED ? 0x54806408u : 0x54006400u;    // 72 / 1032 or 64 / 1024
    constexpr int kLut = SIGNED ? 0x6A : 0xEA;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t x = prmt(w, w, 0x4040u + 0x1111u * (uint32_t)i);   // bytes (i, i, i, i)
        q[i] = h2_sub(lop3<kLut>(x, kMask, kMagic), kBias);
    }
}

// Split K in a cluster: a CTA's fp32 tile in shared memory, rows 257 floats apart.
constexpr int kRedPitch = kBN + 1;

// Per weight format of the single-CTA kernel: INT4 packs 8 K values in a word
// (8 word rows per K step of 64), FP8-E4M3 4 (16 word rows, a twice larger
// packed tile, so one TMA stage fewer fits in shared memory).
template <bool FP8>
struct TcCfg {
    static constexpr int kWordRows = FP8 ? kBK / 4 : kBK / 8;
    static constexpr int kWBytes = kWordRows * kBN * 4;
    static constexpr int kTmaStages = FP8 ? 4 : 5;
    static constexpr int kTmaStageBytes = kABytes + kWBytes + 2 * kSBytes;
    static constexpr int kRingBytes = kTmaStages * kTmaStageBytes + kBStages * kBBytes;
    static constexpr int kBarriers = 2 * kTmaStages + 2 * kBStages + 1;
};

static_assert(kBM * kRedPitch * 4 <= TcCfg<false>::kRingBytes && kBM * kRedPitch * 4 <= TcCfg<true>::kRingBytes,
              "a CTA's fp32 tile fits in its ring");

// Two E4M3 bytes (low byte first) -> fp16x2 (low half first), exactly.
__device__ __forceinline__ uint32_t e4m3x2_to_h2(uint16_t v) {
    uint32_t d;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(d) : "h"(v));
    return d;
}

template <bool SIGNED, bool HAS_ZP, bool FP8>
__global__ void __launch_bounds__(kThreads, 1)
gemm_w4_tc_kernel(const __grid_constant__ GemmMaps maps, const GemmParams p) {
    using C = TcCfg<FP8>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    // TMA slot s: [A 16 KB][packed 8 KB (fp8: 16 KB)][scales 512][zero points 512]; then the B slots (32 KB each)
    uint8_t* bring = base + C::kTmaStages * C::kTmaStageBytes;
    uint64_t* full_tma = reinterpret_cast<uint64_t*>(base + C::kRingBytes);
    uint64_t* empty_tma = full_tma + C::kTmaStages;
    uint64_t* full_b = empty_tma + C::kTmaStages;
    uint64_t* empty_b = full_b + kBStages;
    uint64_t* acc_full = empty_b + kBStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_launch_dependents();     // the next kernel may start its prologue as SMs free up
    const int n0 = blockIdx.x * kBN, m0 = blockIdx.y * kBM;
    const int k_begin = blockIdx.z * p.ks_per;
    const int nsteps = min(p.ks_per, p.ksteps - k_begin);   // >= 1: the host sizes the split so
    volatile int* last_flag = abort_flag + 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kTmaStages; ++s) {
            mbar_init(&full_tma[s], 1);
            mbar_init(&empty_tma[s], 1);          // tcgen05.commit
        }
        for (int s = 0; s < kBStages; ++s) {
            mbar_init(&full_b[s], kDqWarps);      // one arrival per dequant warp
            mbar_init(&empty_b[s], 1);            // tcgen05.commit
        }
        mbar_init(acc_full, 1);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tmap(&maps.a);
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
        // ---------------- TMA producer
        if (lane == 0) {
            // Packed words, scales and zero points are never written by a
            // kernel of this library, so the first ring stages' copies of them
            // go out before the dependency wait on the previous kernel; A's
            // (which that kernel may have written) after it.
            auto weights = [&](int i) {
                const int s = i % C::kTmaStages;
                uint8_t* st = base + s * C::kTmaStageBytes;
                const int kg = k_begin + i;                         // K step in the whole of K
                const int srow = p.gw_steps ? kg / p.gw_steps : 0;
                mbar_arrive_expect_tx(&full_tma[s], kABytes + C::kWBytes + kSBytes * (HAS_ZP ? 2 : 1));
                tma_load_2d(st + kABytes, &maps.w, n0, kg * C::kWordRows, &full_tma[s]);
                tma_load_2d(st + kABytes + C::kWBytes, &maps.s, n0, srow, &full_tma[s]);
                if constexpr (HAS_ZP)
                    tma_load_2d(st + kABytes + C::kWBytes + kSBytes, &maps.z, n0, srow, &full_tma[s]);
            };
            auto act = [&](int i) {
                const int s = i % C::kTmaStages;
                tma_load_2d(base + s * C::kTmaStageBytes, &maps.a, (k_begin + i) * kBK, m0, &full_tma[s]);
            };
            const int pre = min(nsteps, C::kTmaStages);
            for (int i = 0; i < pre; ++i) weights(i);
            pdl_wait_prior_grid();   // A may be the previous kernel's output
            for (int i = 0; i < pre; ++i) act(i);
            for (int i = pre; i < nsteps; ++i) {
                const int s = i % C::kTmaStages;
                const uint32_t ph = (uint32_t)((i / C::kTmaStages) & 1);
                if (!wait_or_abort(&empty_tma[s], ph ^ 1u, abort_flag)) break;
                weights(i);
                act(i);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer
        if (lane == 0) {
            // The dequant warps arrive on full_b[b] only after waiting for the
            // stage's TMA copy, so full_b alone certifies both operands.
            bool ready = mbar_try_wait(&full_b[0], 0);
            for (int i = 0; i < nsteps; ++i) {
                const int s = i % C::kTmaStages, b = i % kBStages;
                if (!ready && !wait_or_abort(&full_b[b], (uint32_t)((i / kBStages) & 1), abort_flag)) break;
                // peek at the next stage while this one's MMAs queue (no tcgen05 fence
                // per stage: the barrier orders the operands, and a fence here would
                // hold the issuer until the queued MMAs drain)
                ready = (i + 1 < nsteps) &&
                        mbar_try_wait(&full_b[(i + 1) % kBStages], (uint32_t)(((i + 1) / kBStages) & 1));
                const uint32_t a_addr = smem_addr(base + s * C::kTmaStageBytes);
                const uint32_t b_addr = smem_addr(bring + b * kBBytes);
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk)
                    tc_mma(tmem_d, smem_desc_sw128(a_addr + kk * 32), smem_desc_sw128(b_addr + kk * 32),
                           (i > 0 || kk > 0) ? 1u : 0u);
                tc_commit(&empty_tma[s]);     // both fire once these MMAs have read their operands
                tc_commit(&empty_b[b]);
            }
            tc_commit(acc_full);     // fires once every MMA issued above has completed
        }
    } else {
        // ---------------- dequant warpgroups (warps 2..17), then epilogue
        const int n = (threadIdx.x - 64) & (kBN - 1);       // column of the tile
        const int j0 = ((threadIdx.x - 64) >> 8) * 4;       // 16-byte units j0 .. j0 + 3 of the K step's B row
        for (int i = 0; i < nsteps; ++i) {
            const int s = i % C::kTmaStages, b = i % kBStages;
            if (!wait_or_abort(&full_tma[s], (uint32_t)((i / C::kTmaStages) & 1), abort_flag)) break;
            if (i >= kBStages && !wait_or_abort(&empty_b[b], (uint32_t)(((i / kBStages) & 1) ^ 1), abort_flag)) break;
            const uint8_t* st = base + s * C::kTmaStageBytes;
            const uint32_t* wp = reinterpret_cast<const uint32_t*>(st + kABytes);
            const uint16_t* sp = reinterpret_cast<const uint16_t*>(st + kABytes + C::kWBytes);
            uint8_t* bt = bring + b * kBBytes;
            const uint16_t sbits = sp[n];
            const uint32_t s2 = h2_dup(sbits);
            float zf = 0.f, sf = 0.f;
            if constexpr (HAS_ZP) {
                zf = h_to_f(sp[kBN + n]);
                sf = h_to_f(sbits);
            }
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                const int j = j0 + jj;       // 16-byte unit = 8 K values: one int4 word or two fp8 words
                if constexpr (FP8) {
                    // E4M3 -> fp16 is exact (subnormals included, NaN stays NaN);
                    // fp16(w * s) is then the contract rounding of the product
                    const uint32_t w0 = wp[(2 * j) * kBN + n], w1 = wp[(2 * j + 1) * kBN + n];
                    uint4 o;
                    o.x = h2_mul(e4m3x2_to_h2((uint16_t)(w0 & 0xFFFFu)), s2);
                    o.y = h2_mul(e4m3x2_to_h2((uint16_t)(w0 >> 16)), s2);
                    o.z = h2_mul(e4m3x2_to_h2((uint16_t)(w1 & 0xFFFFu)), s2);
                    o.w = h2_mul(e4m3x2_to_h2((uint16_t)(w1 >> 16)), s2);
                    *reinterpret_cast<uint4*>(bt + n * 128 + ((j ^ (n & 7)) << 4)) = o;
                    continue;
                }
                const uint32_t w = wp[j * kBN + n];
                uint32_t q[4];
                unpack_natural<SIGNED>(w, q);
                uint4 o;
                uint32_t* ov = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    if constexpr (HAS_ZP) {
                        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&q[k]));
                        ov[k] = f2_to_h2((f.x - zf) * sf, (f.y - zf) * sf);
                    } else {
                        ov[k] = h2_mul(q[k], s2);
                    }
                }
                *reinterpret_cast<uint4*>(bt + n * 128 + ((j ^ (n & 7)) << 4)) = o;
            }
            fence_proxy_async_smem();      // generic-proxy writes of B before the MMA reads them
            __syncwarp();
            if (lane == 0) mbar_arrive(&full_b[b]);
        }
        // ---------------- epilogue: TMEM lanes 32 * (warp % 4) .. +31 = rows of the tile
        pdl_wait_prior_grid();       // before any store: the previous kernel may read or write C
        const bool ok = wait_or_abort(acc_full, 0, abort_flag);
        tc_fence_after();
        const int quarter = warp & 3;                       // TMEM lanes this warp may read
        const int cq = (warp - 2) >> 2;                     // which 64 columns
        const int row = m0 + 32 * quarter + lane;
        if (p.ksplit > 1 && p.cluster_split) {
            // Split K in a cluster: this CTA's fp32 tile goes to its own shared
            // memory -- the ring, idle now (acc_full: every MMA has completed,
            // so every copy has landed and been read) -- as [128][kRedPitch]
            // (pitch 257: the 32 rows a warp writes fall in 32 distinct banks);
            // the peers add the tiles after the cluster barrier below.
            if (ok) {
                float* tile = reinterpret_cast<float*>(base);
                const int r = 32 * quarter + lane;
                for (int c0 = 64 * cq; c0 < 64 * cq + 64; c0 += 32) {
                    uint32_t v[32];
                    tmem_ld32(tmem_d + ((uint32_t)(32 * quarter) << 16) + (uint32_t)c0, v);   // warp-collective
#pragma unroll
                    for (int k = 0; k < 32; ++k) tile[r * kRedPitch + c0 + k] = __uint_as_float(v[k]);
                }
            }
        } else if (p.ksplit > 1) {
            // Split K: this CTA's fp32 tile goes to its partial slot; the last
            // CTA of the tile to arrive adds the ksplit partials in split order
            // -- the same sum whichever CTA is last.  Every
            // dequant warp reaches both barriers (ok may differ per thread after
            // a timeout), and every CTA counts its arrival, so the counter is
            // back at zero when the launch ends even after an abort (whose
            // output is then wrong, and flagged in the error word).
            const int tile = blockIdx.y * gridDim.x + blockIdx.x;
            const int r = 32 * quarter + lane;
            float* mine = p.part + (((size_t)tile * p.ksplit + blockIdx.z) * kBM + r) * kBN;
            if (ok) {
                for (int c0 = 64 * cq; c0 < 64 * cq + 64; c0 += 32) {
                    uint32_t v[32];
                    // warp-collective: every lane loads, whatever its row
                    tmem_ld32(tmem_d + ((uint32_t)(32 * quarter) << 16) + (uint32_t)c0, v);
                    // rows past M (a decode batch fills one row of 128) are
                    // neither stored nor summed
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
            if (threadIdx.x == 64) {
                const bool last = atomicAdd(p.counters + tile, 1u) == (unsigned)(p.ksplit - 1);
                if (last) p.counters[tile] = 0u;     // every CTA of the tile has arrived
                *last_flag = last ? 1 : 0;
                __threadfence();
            }
            asm volatile("bar.sync 1, %0;" ::"n"(32 * kDqWarps) : "memory");
            if (ok && *last_flag != 0) {
                // Every partial (this CTA's too) is in the workspace: sum the
                // tile flat, consecutive threads on consecutive float4s (fully
                // coalesced), four splits' loads in flight, in split order.
                const int t = threadIdx.x - 64;                  // 0 .. 511
                constexpr int kPer = kBM * kBN / 4;              // float4s in a partial
                const int valid = min(kBM, p.M - m0) * (kBN / 4);   // float4s of the tile's rows < M
                const float4* src = reinterpret_cast<const float4*>(p.part) + (size_t)tile * p.ksplit * kPer;
                for (int i = t; i < valid; i += 32 * kDqWarps) {
                    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                    for (int z0 = 0; z0 < p.ksplit; z0 += 4) {
                        float4 f[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u)
                            f[u] = (z0 + u < p.ksplit) ? __ldcg(src + (size_t)(z0 + u) * kPer + i)
                                                       : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            acc.x += f[u].x; acc.y += f[u].y; acc.z += f[u].z; acc.w += f[u].w;
                        }
                    }
                    const int gr = m0 + (i >> 6), gc = n0 + ((i & 63) << 2);   // 64 float4s a row
                    if (gr < p.M && gc < p.N) {       // N % 8 == 0: a float4 is all in or all out
                        uint2 o;
                        o.x = f2_to_h2(acc.x, acc.y);
                        o.y = f2_to_h2(acc.z, acc.w);
                        *reinterpret_cast<uint2*>(p.C + (size_t)gr * p.N + gc) = o;
                    }
                }
            }
        } else if (ok) {
            for (int c0 = 64 * cq; c0 < 64 * cq + 64; c0 += 32) {
                uint32_t v[32];
                tmem_ld32(tmem_d + ((uint32_t)(32 * quarter) << 16) + (uint32_t)c0, v);
                if (row < p.M) {
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
        if (warp >= 2 && !*abort_flag) {
            // CTA `rank` adds, for its share of the tile's elements (rows < M
            // only, row-major, consecutive threads on consecutive columns), the
            // ksplit tiles in split order -- the same sum on every run.
            const int ks = p.ksplit;
            const int rank = (int)cluster_rank();
            const int rows = min(kBM, p.M - m0);
            const int E = rows * kBN;
            const int per = (E + ks - 1) / ks;
            const int e_end = min(E, (rank + 1) * per);
            const uint32_t tile0 = smem_addr(base);
            uint32_t peer[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) peer[q] = q < ks ? map_to_rank(base, (uint32_t)q) : tile0;
            for (int e = rank * per + (int)threadIdx.x - 64; e < e_end; e += 32 * kDqWarps) {
                const int r = e >> 8, c = e & (kBN - 1);
                const uint32_t off = (uint32_t)(r * kRedPitch + c) * 4u;
                float v = 0.f;
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    if (q < ks) v += ld_dsmem_f32(peer[q] + off);
                if (n0 + c < p.N) p.C[(size_t)(m0 + r) * p.N + n0 + c] = __half_as_ushort(__float2half_rn(v));
            }
        }
        cluster_sync_all();      // no CTA leaves while a peer still reads its tile
    }

    // ---------------- teardown: no MMA may still be writing TMEM when it is freed
    tc_fence_before();
    __syncthreads();
    if (*abort_flag && threadIdx.x == 32) {
        // the issuer committed acc_full after its last MMA; wait for it (bounded)
        mbar_wait_bounded(acc_full, 0, kWaitLimitNs / 4);
        // and for copies still landing in the ring
        for (int s = 0; s < C::kTmaStages; ++s) mbar_wait_bounded(&full_tma[s], 0, kWaitLimitNs / 8);
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(kBN));
    }
}

// =============================================================================
// CTA-pair variant (M > 128): a cluster of two CTAs on one TPC runs
// tcgen05.mma.cta_group::2 with M = 256, N = 256 -- the pair computes a
// 256 x 256 tile of C, each CTA holding its 128 rows of A and dequantizing 128
// of the 256 weight columns (the MMA takes the B operand N-split across the
// two CTAs' shared memory at the same offset).  Against the single-CTA
// kernel this halves the dequant work and the shared-memory traffic of B per
// SM (B is the largest operand there), which is what bounds that kernel.
//
//   warp 0      (both CTAs) one thread issues this CTA's TMA copies of a
//               stage (A 128 x 64, packed words 8 x 128, one scale row) and
//               signals this CTA's own "full" barrier -- no copy writes or
//               signals the other CTA;
//   warp 1      (both CTAs) allocates the pair's TMEM (cta_group::2); in the
//               leader CTA one thread waits for the pair's B slot to be
//               complete, issues the four K = 16 MMAs of the stage and commits
//               them to the "done" barrier of the stage in BOTH CTAs (two
//               commits, one per CTA, no multicast);
//   warps 2..   dequantize this CTA's 128 columns into its B slot, then arrive
//               on the LEADER's "B full" barrier (a cluster-scope remote arrive
//               from the other CTA).  Their arrival also certifies the stage's
//               A copy, which they waited for, so the issuer waits on one
//               barrier per stage.  After the last stage they drain this CTA's
//               128 accumulator rows from TMEM.
// "done[s]" frees TMA slot s (stage i reuses it after stage i - kPairTmaStages)
// and B slot (i - kPairBStages) % kPairBStages.
namespace pair {

constexpr int kRows = 128;                          // rows of A per CTA
constexpr int kCols = 256;                          // columns of C per pair
constexpr int kHalf = 128;                          // B columns per CTA
constexpr int kTmaStages = 6;
constexpr int kBStages = 4;
constexpr int kDqWarps = 8;
constexpr int kThreads = 64 + 32 * kDqWarps;
constexpr int kWordsPerThread = 8 * kHalf / (32 * kDqWarps);   // packed words (of the 8 per column) per thread
constexpr int kABytes = kRows * kBK * 2;            // 16 KB
constexpr int kWBytes = (kBK / 8) * kHalf * 4;      // 4 KB
constexpr int kSBytes = kHalf * 2;                  // 256 B
constexpr int kStageBytes = 21 * 1024;              // A, packed, scales, zero points, padded so every A tile is 1024-aligned
constexpr int kBBytes = kHalf * kBK * 2;            // 16 KB
constexpr int kRingBytes = kTmaStages * kStageBytes + kBStages * kBBytes;
constexpr int kBarriers = 2 * kTmaStages + kBStages + 1;
static_assert(kWordsPerThread * 32 * kDqWarps == 8 * kHalf, "dequant split");
static_assert(kTmaStages > kBStages, "done-barrier reuse argument needs more TMA stages than B stages");
static_assert(kStageBytes % 1024 == 0 && kStageBytes >= kABytes + kWBytes + 2 * kSBytes, "stage layout");
static_assert((kTmaStages * kStageBytes) % 1024 == 0 && kBBytes % 1024 == 0, "B slots 1024-aligned");

// kind::f16, fp16 A/B K-major, fp32 accumulator, M = 256 (pair), N = 256.
constexpr uint32_t kInstrDesc = tc_idesc_f16(2 * kRows, kCols);

// Bounded wait; the fast path is a single try_wait.
__device__ __forceinline__ bool wait_pair(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (global_timer_ns() - t0 > kWaitLimitNs) break;
    }
    *abort_flag = 1;
    atomicOr(&g_gemm_tc_error, kErrTimeout);
    return false;
}

__device__ __forceinline__ void mma_pair(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
    tc_mma_pair_f16(tmem_d, da, db, kInstrDesc, accumulate);
}

template <bool SIGNED, bool HAS_ZP>
__global__ void __launch_bounds__(kThreads, 1)
gemm_w4_tc_pair_kernel(const __grid_constant__ GemmMaps maps, const GemmParams p) {
    extern __shared__ uint8_t smem_raw[];
    // Same offsets in both CTAs: the MMA addresses the partner's operands by
    // this CTA's shared-memory offsets.
    uint8_t* base = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    uint8_t* bring = base + kTmaStages * kStageBytes;
    uint64_t* full_tma = reinterpret_cast<uint64_t*>(base + kRingBytes);
    uint64_t* done = full_tma + kTmaStages;
    uint64_t* full_b = done + kTmaStages;            // used in the leader only
    uint64_t* acc_full = full_b + kBStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_launch_dependents();     // the next kernel may start its prologue as SMs free up
    const uint32_t rank = cluster_rank();            // 0 = leader (issues the MMAs)
    // 1-D grid of pairs (clusters of 2 along x), column tiles fastest
    const int pair_id = blockIdx.x >> 1;
    const int n_tiles = (p.N + kCols - 1) / kCols;
    const int n0 = (pair_id % n_tiles) * kCols;      // pair's columns
    const int nh = n0 + (int)rank * kHalf;           // this CTA's B columns
    const int m0 = (pair_id / n_tiles) * (2 * kRows) + (int)rank * kRows;   // this CTA's rows
    // split K (gridDim.y splits): this pair's K steps [k_begin, k_begin + nsteps)
    const int k_begin = blockIdx.y * p.ks_per;
    const int nsteps = min(p.ks_per, p.ksteps - k_begin);   // >= 1: the host sizes the split so
    volatile int* last_flag = abort_flag + 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kTmaStages; ++s) {
            mbar_init(&full_tma[s], 1);
            mbar_init(&done[s], 1);              // one commit from the leader's issuer
        }
        for (int b = 0; b < kBStages; ++b) mbar_init(&full_b[b], 2 * kDqWarps);   // every dequant warp of the pair
        mbar_init(acc_full, 1);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tmap(&maps.a);
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
        // ---------------- TMA producer (each CTA loads only its own operands)
        if (lane == 0) {
            // the weights of the first ring stages before the dependency wait,
            // A after it (as in the single-CTA kernel)
            auto weights = [&](int i) {
                const int s = i % kTmaStages;
                uint8_t* st = base + s * kStageBytes;
                const int kg = k_begin + i;                         // K step in the whole of K
                const int srow = p.gw_steps ? kg / p.gw_steps : 0;
                mbar_arrive_expect_tx(&full_tma[s], kABytes + kWBytes + kSBytes * (HAS_ZP ? 2 : 1));
                tma_load_2d(st + kABytes, &maps.w, nh, kg * (kBK / 8), &full_tma[s]);
                tma_load_2d(st + kABytes + kWBytes, &maps.s, nh, srow, &full_tma[s]);
                if constexpr (HAS_ZP)
                    tma_load_2d(st + kABytes + kWBytes + kSBytes, &maps.z, nh, srow, &full_tma[s]);
            };
            auto act = [&](int i) {
                const int s = i % kTmaStages;
                tma_load_2d(base + s * kStageBytes, &maps.a, (k_begin + i) * kBK, m0, &full_tma[s]);
            };
            const int pre = min(nsteps, kTmaStages);
            for (int i = 0; i < pre; ++i) weights(i);
            pdl_wait_prior_grid();   // A may be the previous kernel's output
            for (int i = 0; i < pre; ++i) act(i);
            for (int i = pre; i < nsteps; ++i) {
                if (!wait_pair(&done[i % kTmaStages], (uint32_t)(((i / kTmaStages) & 1) ^ 1), abort_flag)) break;
                weights(i);
                act(i);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (leader CTA only)
        if (rank == 0 && lane == 0) {
            // cluster addresses of done[0] in each CTA; done[s] lies 8 s bytes further
            const uint32_t done0 = map_to_rank(&done[0], 0), done1 = map_to_rank(&done[0], 1);
            bool ready = mbar_try_wait(&full_b[0], 0);
            for (int i = 0; i < nsteps; ++i) {
                const int s = i % kTmaStages, b = i % kBStages;
                if (!ready && !wait_pair(&full_b[b], (uint32_t)((i / kBStages) & 1), abort_flag)) break;
                // peek at the next stage while this one's MMAs queue (no tcgen05 fence
                // per stage: the barrier orders the operands, and a fence here would
                // hold the issuer until the queued MMAs drain)
                ready = (i + 1 < nsteps) &&
                        mbar_try_wait(&full_b[(i + 1) % kBStages], (uint32_t)(((i + 1) / kBStages) & 1));
                const uint32_t a_addr = smem_addr(base + s * kStageBytes);
                const uint32_t b_addr = smem_addr(bring + b * kBBytes);
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk)
                    mma_pair(tmem_d, smem_desc_sw128(a_addr + kk * 32), smem_desc_sw128(b_addr + kk * 32),
                             (i > 0 || kk > 0) ? 1u : 0u);
                commit_pair(done0 + (uint32_t)(s * 8));     // fire once these MMAs have read their operands
                commit_pair(done1 + (uint32_t)(s * 8));
            }
            commit_pair(map_to_rank(acc_full, 0));     // fire once every MMA issued above has completed
            commit_pair(map_to_rank(acc_full, 1));
        }
    } else {
        // ---------------- dequant warps, then epilogue
        const int t = threadIdx.x - 64;
        const int n = t & (kHalf - 1);                       // column of this CTA's half
        const int j0 = (t / kHalf) * kWordsPerThread;        // first word row of the K step
        const uint32_t full_b_leader = map_to_rank(&full_b[0], 0);
        for (int i = 0; i < nsteps; ++i) {
            const int s = i % kTmaStages, b = i % kBStages;
            if (!wait_pair(&full_tma[s], (uint32_t)((i / kTmaStages) & 1), abort_flag)) break;
            if (i >= kBStages) {
                const int r = i - kBStages;
                if (!wait_pair(&done[r % kTmaStages], (uint32_t)((r / kTmaStages) & 1), abort_flag)) break;
            }
            const uint8_t* st = base + s * kStageBytes;
            const uint32_t* wp = reinterpret_cast<const uint32_t*>(st + kABytes);
            const uint16_t* sp = reinterpret_cast<const uint16_t*>(st + kABytes + kWBytes);
            uint8_t* bt = bring + b * kBBytes;
            const uint16_t sbits = sp[n];
            const uint32_t s2 = h2_dup(sbits);
            float zf = 0.f, sf = 0.f;
            if constexpr (HAS_ZP) {
                zf = h_to_f(sp[kHalf + n]);
                sf = h_to_f(sbits);
            }
#pragma unroll
            for (int jj = 0; jj < kWordsPerThread; ++jj) {
                const int j = j0 + jj;
                const uint32_t w = wp[j * kHalf + n];
                uint32_t q[4];
                unpack_natural<SIGNED>(w, q);
                uint4 o;
                uint32_t* ov = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    if constexpr (HAS_ZP) {
                        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&q[k]));
                        ov[k] = f2_to_h2((f.x - zf) * sf, (f.y - zf) * sf);
                    } else {
                        ov[k] = h2_mul(q[k], s2);
                    }
                }
                *reinterpret_cast<uint4*>(bt + n * 128 + ((j ^ (n & 7)) << 4)) = o;
            }
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
        const int cq = (warp - 2) >> 2;
        const int row = m0 + 32 * quarter + lane;
        if (p.ksplit > 1) {
            // Split K, as in the single-CTA kernel, per CTA: this CTA's 128 rows
            // x 256 columns go to their partial slot; the last of the ksplit
            // CTAs holding these rows sums the partials in split order (flat,
            // coalesced) and writes C.  Every dequant warp reaches both
            // barriers, and every CTA counts its arrival.
            const int tile = 2 * pair_id + (int)rank;
            const int r = 32 * quarter + lane;
            float* mine = p.part + (((size_t)tile * p.ksplit + blockIdx.y) * kRows + r) * kCols;
            if (ok) {
                for (int c0 = kColsPerWarp * cq; c0 < kColsPerWarp * cq + kColsPerWarp; c0 += 32) {
                    uint32_t v[32];
                    tmem_ld32(tmem_d + ((uint32_t)(32 * quarter) << 16) + (uint32_t)c0, v);
#pragma unroll
                    for (int k = 0; k < 32; k += 4)
                        __stcg(reinterpret_cast<float4*>(mine + c0 + k),
                               make_float4(__uint_as_float(v[k]), __uint_as_float(v[k + 1]),
                                           __uint_as_float(v[k + 2]), __uint_as_float(v[k + 3])));
                }
            }
            __threadfence();
            asm volatile("bar.sync 1, %0;" ::"n"(32 * kDqWarps) : "memory");
            if (threadIdx.x == 64) {
                const bool last = atomicAdd(p.counters + tile, 1u) == (unsigned)(p.ksplit - 1);
                if (last) p.counters[tile] = 0u;     // every CTA holding these rows has arrived
                *last_flag = last ? 1 : 0;
                __threadfence();
            }
            asm volatile("bar.sync 1, %0;" ::"n"(32 * kDqWarps) : "memory");
            if (ok && *last_flag != 0) {
                const int t2 = threadIdx.x - 64;                  // 0 .. 255
                constexpr int kPer = kRows * kCols / 4;           // float4s in a partial
                constexpr int kRow4 = kCols / 4;
                const float4* src = reinterpret_cast<const float4*>(p.part) + (size_t)tile * p.ksplit * kPer;
                for (int i = t2; i < kPer; i += 32 * kDqWarps) {
                    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                    for (int z0 = 0; z0 < p.ksplit; z0 += 4) {
                        float4 f[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u)
                            f[u] = (z0 + u < p.ksplit) ? __ldcg(src + (size_t)(z0 + u) * kPer + i)
                                                       : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            acc.x += f[u].x; acc.y += f[u].y; acc.z += f[u].z; acc.w += f[u].w;
                        }
                    }
                    const int gr = m0 + i / kRow4, gc = n0 + (i % kRow4) * 4;
                    if (gr < p.M && gc < p.N) {       // N % 8 == 0: a float4 is all in or all out
                        uint2 o;
                        o.x = f2_to_h2(acc.x, acc.y);
                        o.y = f2_to_h2(acc.z, acc.w);
                        *reinterpret_cast<uint2*>(p.C + (size_t)gr * p.N + gc) = o;
                    }
                }
            }
        } else if (ok) {
            for (int c0 = kColsPerWarp * cq; c0 < kColsPerWarp * cq + kColsPerWarp; c0 += 32) {
                uint32_t v[32];
                tmem_ld32(tmem_d + ((uint32_t)(32 * quarter) << 16) + (uint32_t)c0, v);
                if (row < p.M) {
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
        // the leader's issuer committed acc_full after its last MMA; wait for it (bounded)
        mbar_wait_bounded(acc_full, 0, kWaitLimitNs / 4);
        for (int s = 0; s < kTmaStages; ++s) mbar_wait_bounded(&full_tma[s], 0, kWaitLimitNs / 8);
    }
    __syncthreads();
    cluster_sync_all();          // neither CTA frees TMEM or exits while the other may still signal it
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(kCols));
    }
}

template <bool SIGNED, bool HAS_ZP>
int launch(const GemmMaps& maps, const GemmParams& p, cudaStream_t stream) {
    auto kern = gemm_w4_tc_pair_kernel<SIGNED, HAS_ZP>;
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

template <bool SIGNED, bool HAS_ZP, bool FP8 = false>
int launch(const GemmMaps& maps, const GemmParams& p, cudaStream_t stream) {
    using C = TcCfg<FP8>;
    auto kern = gemm_w4_tc_kernel<SIGNED, HAS_ZP, FP8>;
    const size_t smem = 1024 + (size_t)C::kRingBytes + C::kBarriers * 8 + 16;
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

// How many clusters of `ks` single-CTA GEMM CTAs can be resident at once on
// the current device: a cluster must fit in one GPC, so large clusters of
// one-CTA-per-SM kernels fit fewer times than the SM count suggests
// (measured: 16 clusters of 8 ran in two waves).
int cluster_capacity(int ks) {
    using C = TcCfg<false>;
    static ClusterCapacityCache cache;
    return max_active_clusters(reinterpret_cast<const void*>(gemm_w4_tc_kernel<true, false, false>),
                               1024 + C::kRingBytes + C::kBarriers * 8 + 16, kThreads, ks, &cache);
}

// The largest split of `tiles` single-CTA tiles into clusters of at most `ks`
// that are all resident at once (1: none).
int cluster_split_of(int tiles, int ks) {
    for (; ks >= 2; --ks)
        if (tiles <= cluster_capacity(ks)) return ks;
    return 1;
}

}  // namespace

int gemm_tc_device_error(cudaStream_t stream, unsigned* out, bool clear) {
    unsigned* word = nullptr;
    cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&word), g_gemm_tc_error);
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, word, sizeof(unsigned), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess && clear) e = cudaMemsetAsync(word, 0, sizeof(unsigned), stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    return e == cudaSuccess ? T4B_OK : record_cuda_error(e);
}

int gemm_w4_tc(bool is_signed, const void* A, const void* W, const void* S, const void* Z, void* C, int M, int N, int K,
               int group, bool allow_pairs, cudaStream_t stream) {
    if (M <= 16 || (K % kBK) != 0 || (group % kBK) != 0 || (N % 8) != 0) return T4B_ERR_UNSUPPORTED;
    if (!aligned(A, 16) || !aligned(W, 16) || !aligned(S, 16) || (Z && !aligned(Z, 16)) || !aligned(C, 16))
        return T4B_ERR_UNSUPPORTED;
    GemmParams p;
    p.C = static_cast<uint16_t*>(C);
    p.M = M; p.N = N; p.K = K;
    p.ksteps = K / kBK;
    p.gw_steps = (group >= K) ? 0 : group / kBK;
    p.ksplit = 1;
    p.ks_per = p.ksteps;
    p.cluster_split = 0;
    p.part = nullptr;
    p.counters = nullptr;
    // M > 128: CTA pairs (each CTA dequantizes 128 of a pair's 256 columns).
    // When the tiles (or pairs) leave SMs idle and K is long, K is split
    // across CTAs (or pairs) until about one CTA per SM (at least 8 K steps a
    // split).  Measured: gains at K >= 8192, but losses at K = 4096 with a
    // third or more of the SMs busy, where storing and re-reading the fp32
    // partials costs more than the idle SMs.
    bool use_pair = M > kBM && allow_pairs;
    const int sms = sm_count();
    const int tiles = ((M + kBM - 1) / kBM) * ((N + kBN - 1) / kBN);
    const int pair_ctas = 2 * ((M + 2 * kBM - 1) / (2 * kBM)) * ((N + kBN - 1) / kBN);
    // Below K = 8192 a grid of at most a quarter of the SMs splits from 8 K
    // steps a split, one of at most half the SMs from 16 (single CTAs, whose
    // splits add up in a cluster; measured at M = 512: 4096 x 1024 168 -> 247
    // TFLOP/s, 4096 x 4096 541 -> 617; at 8 K steps a split of a 64-tile grid
    // the cluster's fixed cost lost, 323 -> 279).
    const bool long_k = p.ksteps >= kMinSplitK / kBK;
    const bool quarter = 4 * tiles <= sms;
    if ((long_k || 2 * tiles <= sms) && tiles < sms && (!use_pair || pair_ctas < sms)) {
        const int min_steps = (long_k || quarter) ? kMinSplitSteps : kMinLooseSplitSteps;
        auto split_of = [&](int ctas) { return std::min(std::min(sms / ctas, p.ksteps / min_steps), 8); };
        // M > 128 splits the CTA pairs (half a single CTA's dequant per SM)
        // when each split keeps a long K run; with short runs the pair's
        // larger fixed cost wins out (measured against single CTAs: +5-10 % at
        // 224 K steps a split, +1-3 % at 112, -2-10 % at 64, -16 % at 16), and
        // single CTAs split instead.  Either way a partial
        // is one CTA's 128 x 256 accumulator.
        if (use_pair) {
            const int kp = (long_k || quarter) ? split_of(pair_ctas) : 1;
            const bool pair_split = kp >= 2 && (p.ksteps + kp - 1) / kp >= kMinPairSplitSteps;
            if (!pair_split && cluster_split_of(tiles, split_of(tiles)) >= 2) use_pair = false;
        }
        const int ctas = use_pair ? pair_ctas : tiles;
        const int ks = use_pair ? split_of(ctas) : cluster_split_of(tiles, split_of(tiles));
        if (ks >= 2 && !use_pair) {
            // single CTAs: the splits of a tile are one cluster and add their
            // tiles through distributed shared memory (no workspace)
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
    const uint32_t wbox = use_pair ? pair::kHalf : kBN;
    GemmMaps maps;
    if (!make_tmap_2d_ex(&maps.a, true, A, (uint64_t)M, (uint64_t)K, kBM, kBK, 128, 256) ||
        !make_tmap_2d_ex(&maps.w, false, W, (uint64_t)(K / 8), (uint64_t)N, kBK / 8, wbox, 0, 256) ||
        !make_tmap_2d_ex(&maps.s, true, S, (uint64_t)(K / group), (uint64_t)N, 1, wbox, 0, 0))
        return T4B_ERR_UNSUPPORTED;
    if (Z) {
        if (!make_tmap_2d_ex(&maps.z, true, Z, (uint64_t)(K / group), (uint64_t)N, 1, wbox, 0, 0))
            return T4B_ERR_UNSUPPORTED;
    } else {
        maps.z = maps.s;
    }
    if (use_pair) {
        if (is_signed) return Z ? pair::launch<true, true>(maps, p, stream) : pair::launch<true, false>(maps, p, stream);
        return Z ? pair::launch<false, true>(maps, p, stream) : pair::launch<false, false>(maps, p, stream);
    }
    if (is_signed) return Z ? launch<true, true>(maps, p, stream) : launch<true, false>(maps, p, stream);
    return Z ? launch<false, true>(maps, p, stream) : launch<false, false>(maps, p, stream);
}

// FP8-E4M3 weights (4 per word, K row 4 kw + j in byte j of word (kw, n)),
// fp16 activations: the single-CTA kernel with the E4M3 dequant, for every M
// (a decode batch fills one 128-row tile).  Where the tiles leave SMs idle, K
// is split as in the INT4 GEMM, here from 4 K steps a split: at small M the
// dequant of B, which every split shares evenly, is the whole cost.
int gemm_fp8_tc(const void* A, const void* W, const void* S, void* C, int M, int N, int K, int group,
                cudaStream_t stream) {
    using Cfg = TcCfg<true>;
    if (M < 1 || (K % kBK) != 0 || (group % kBK) != 0 || (N % 8) != 0) return T4B_ERR_UNSUPPORTED;
    if (!aligned(A, 16) || !aligned(W, 16) || !aligned(S, 16) || !aligned(C, 16)) return T4B_ERR_UNSUPPORTED;
    GemmParams p;
    p.C = static_cast<uint16_t*>(C);
    p.M = M; p.N = N; p.K = K;
    p.ksteps = K / kBK;
    p.gw_steps = (group >= K) ? 0 : group / kBK;
    p.ksplit = 1;
    p.ks_per = p.ksteps;
    p.cluster_split = 0;
    p.part = nullptr;
    p.counters = nullptr;
    const int sms = sm_count();
    const int tiles = ((M + kBM - 1) / kBM) * ((N + kBN - 1) / kBN);
    const int ks = cluster_split_of(tiles, std::min(std::min(sms / tiles, p.ksteps / 4), 8));
    if (ks >= 2) {
        p.ks_per = (p.ksteps + ks - 1) / ks;
        p.ksplit = (p.ksteps + p.ks_per - 1) / p.ks_per;      // no empty split
        p.cluster_split = 1;                                  // a cluster of splits per tile
    }
    GemmMaps maps;
    if (!make_tmap_2d_ex(&maps.a, true, A, (uint64_t)M, (uint64_t)K, kBM, kBK, 128, 256) ||
        !make_tmap_2d_ex(&maps.w, false, W, (uint64_t)(K / 4), (uint64_t)N, Cfg::kWordRows, kBN, 0, 256) ||
        !make_tmap_2d_ex(&maps.s, true, S, (uint64_t)(K / group), (uint64_t)N, 1, kBN, 0, 0))
        return T4B_ERR_UNSUPPORTED;
    maps.z = maps.s;
    return launch<true, false, true>(maps, p, stream);
}

}  // namespace t4b

extern "C" int t4b_fused_w8a16_gemm_fp8(const void* A, const void* W_packed, const void* scales, void* C, int M,
                                        int N, int K, int group_size, void* stream) {
    using namespace t4b;
    if (M < 1 || N < 1 || K < 4 || (K % 4) != 0) return T4B_ERR_INVALID_VALUE;
    if (group_size < 4 || (K % group_size) != 0) return T4B_ERR_INVALID_VALUE;
    if (!A || !W_packed || !scales || !C) return T4B_ERR_NULL_POINTER;
    if (!aligned(A, 16) || !aligned(W_packed, 16) || !aligned(scales, 16) || !aligned(C, 16)) return T4B_ERR_MISALIGNED;
    return gemm_fp8_tc(A, W_packed, scales, C, M, N, K, group_size, static_cast<cudaStream_t>(stream));
}
