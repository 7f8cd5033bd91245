// Decode W4A16 GEMV with the activations resident in shared memory:
//
//   C[M, N] = A[M, K] x dequant(W)[K, N],  W int32 [K/8, N], group scales [K/g, N]
//
// for M <= 16 (one token, or a handful, per call) whose activations fit in
// shared memory next to a ring of at least two stages; past M * K = 32768 only
// for shapes with at least one 16-column tile per SM.
//
// Work decomposition
//   Output columns are cut into 16-column tiles.  CTA b of G (G <= SMs) owns
//   the contiguous tiles [b T / G, (b+1) T / G) over the whole of K, so no two
//   CTAs ever produce the same output: there is no cross-CTA traffic and no
//   wait on another CTA.  A CTA walks its tiles in groups of up to four
//   (64 columns); each group streams its weight columns over K through a
//   ring of shared-memory stages and ends with one reduction across warps.
//
// Stages
//   A CTA has WARPS warps (16 for M <= 8, else 8) and a stage gives each warp
//   16 word rows x 32 columns: one TMA box per 16-column tile of the group,
//   covering all the stage's rows (8 * WARPS rows for groups of 3-4 tiles,
//   16 * WARPS rows for groups of 1-2; 64-byte swizzle), plus one box of
//   group scales (and one of zero points) over the stage's rows and the
//   group's 64 or 32 columns -- a handful of large copies per stage, because the
//   thread that issues a copy stalls while the SM's copy engine is busy.
//   All of it is constant data, so every stage the ring holds is issued at
//   kernel entry, before griddepcontrol.wait, and streams in while the
//   previous kernel in the stream drains.  One CTA fills an SM: a ring as
//   deep as shared memory allows keeps ~200 KB per SM in flight, which the
//   copy engine needs to stream 64-byte box rows at full rate (measured in
//   the decode step: 1.62 ms against 2.24 ms with two co-resident CTAs of
//   half the depth).  A dedicated producer warp refills the slots: a copy
//   issue can stall for hundreds of cycles while the copy engine is busy, and
//   a math warp doing it would put that stall on every stage's critical path.
//   The math warps release a slot by arriving on its "empty" barrier.
//
// Activations
//   After griddepcontrol.wait the CTA copies A into shared memory once, as one
//   16-byte record (a0,a4),(a1,a5),(a2,a6),(a3,a7) per batch row and 8-element
//   word row -- exactly the B fragment of mma.m16n8k16 that the unpacked
//   weights below need -- and sums every batch row over each flush block of 8
//   or 16 word rows.
//
// Math
//   Warp (wc, rb) owns 32 columns (two 16-column boxes) x 16 word rows of a
//   stage.  A lane reads four words of one row (one 16-byte load) and turns
//   each into four fp16x2 registers with one LOP3 per nibble pair (0,4),
//   (1,5), (2,6), (3,7): the pair lands in mantissa bits 4-7 under exponent
//   2^6, which reads exactly as 64 + u (unsigned) or, with the nibble's top
//   bit flipped, 72 + s (signed).  These offset integers are the A operand of
//   mma.m16n8k16 with fp32 accumulation; per flush block the offset leaves
//   with the activation sum:
//       y += scale * (sum (o + q) a  -  (o + z) sum a),   o = 64 or 72.
#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "tma.cuh"

namespace t4b {
namespace {

constexpr int kBoxCols = 16;                       // columns per TMA box (64 bytes)
constexpr int kMaxStages = 12;
constexpr int kMaxProj = T4B_GROUPED_MAX;          // projections of one grouped launch
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr unsigned kErrTimeout = 1u;

template <int MT>
struct Shape {
    static constexpr int kWarps = (MT == 1) ? 16 : 8;          // consumer (math) warps
    static constexpr int kThreads = 32 * (kWarps + 1);         // + one producer warp
    static constexpr int kWeightBytes = kWarps * 2048;         // packed words per stage
    static constexpr int kRowsNarrow = 16 * kWarps;            // stage rows, 1 warp column (1-2 tiles)
    static constexpr int kRowsWide = 8 * kWarps;               // stage rows, 2 warp columns (4 tiles)
    static constexpr int kRowsSplit = 32 * kWarps;             // stage rows of a split group (1 tile, two row halves)
};

// Device error word of this kernel (bit 0: a bounded wait gave up), one per
// device.  Device code sets it by name, so a call needs no workspace and can
// be captured into a CUDA graph on any stream; decode_device_error() reads it.
__device__ unsigned g_decode_error = 0;

struct DecodeParams {
    const uint16_t* A;
    uint16_t* C;
    int M, N, K, KW;
    int KWp;            // word rows padded to a multiple of the narrow stage (resident activations)
    int T, G;           // 16-column tiles, CTAs
    int gw;             // group size in word rows
    int gw_shift;       // log2(gw) when gw is a power of two (it then divides any stage it is smaller than)
    int fb;             // flush block in word rows: 8 (gw == 8) or 16
    int sbr_wide;       // scale rows of a wide stage's scale box: rows_wide / gw, or 1 when gw >= rows_wide
    int sbr_narrow;     // same for a narrow stage
    int s_bytes;        // bytes of the scale (and of the zero-point) region of a slot
    int stages;         // ring depth
    int early;          // stages issued before griddepcontrol.wait (the rest right after it)
    int slot_bytes;     // bytes of one ring slot
    int s_wide, s_narrow;   // stages of a wide (4-tile) / narrow (1-2 tile) group
    int split;          // a lone tile streams as a split group (M <= 4; see cta_plan)
    int s_split;        // stages of a split group
    int sbr_split;      // scale rows of a split stage's scale box
    int act_bytes;      // resident activation records (bytes)
    int sum_floats;     // flush-block activation sums
    int red_floats;     // cross-warp reduction buffer
    FastDiv kwdiv;      // division by KWp
    // Projections of this launch (one, or a group that shares A): projection
    // j owns CTAs [proj_g0[j], proj_g0[j+1]) and its T = proj_T[j] tiles,
    // output proj_C[j] of proj_N[j] columns.  T and G above are the launch's
    // totals (the grid is G CTAs), N and C those of projection 0.
    int nproj;
    int proj_g0[kMaxProj + 1];
    int proj_T[kMaxProj];
    int proj_N[kMaxProj];
    uint16_t* proj_C[kMaxProj];
    int proj_coloff[kMaxProj];  // fused all-gather: first column of each projection in the group buffer
    // fused all-gather (world > 1): each pair of output columns goes, with the
    // call's epoch, as one 64-bit word to every rank's receive buffer
    unsigned long long* recv[8];
    uint32_t* gout;         // this rank's gathered output (column pairs)
    unsigned* counter;      // [0] CTAs of a group's last launch done, [1] groups done
    int world, rank, n_total, col_offset, barrier;
};

// Tensor maps of one projection.
struct ProjMaps {
    CUtensorMap w_wide;     // packed words, box 16 columns x rows_wide
    CUtensorMap w_narrow;   // packed words, box 16 columns x rows_narrow
    CUtensorMap s_wide;     // scales, box 64 columns x sbr_wide rows
    CUtensorMap s_narrow;   // scales, box 32 columns x sbr_narrow rows
    CUtensorMap z_wide;     // zero points, same boxes (unused without them)
    CUtensorMap z_narrow;
    CUtensorMap s_split;    // scales, box 16 columns x sbr_split rows
    CUtensorMap z_split;
};

template <int NP>
struct DecodeMaps {
    ProjMaps proj[NP];
};

// A pure function of its operands (not volatile), so the compiler may
// interleave independent MMAs with the loads and unpacking around them.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Same with a zero accumulator in (the first MMA of a flush block).
__device__ __forceinline__ void mma_16816_zero(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
    const float z = 0.f;
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
}

// Shared-memory loads by 32-bit address.  Not volatile (free to interleave
// with the math), but with a memory clobber so they stay after the mbarrier
// wait that makes the data visible.
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr) : "memory");
    return v;
}

__device__ __forceinline__ float lds32f(uint32_t addr) {
    float v;
    asm("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

__device__ __forceinline__ uint2 lds64(uint32_t addr) {
    uint2 v;
    asm("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr) : "memory");
    return v;
}

// 32-bit integer multiplies: the low word for a left shift and the high word
// for a right shift by a constant.  They issue to the FMA pipe, while shifts
// and LOP3 share the integer pipe, which the unpacking below otherwise
// saturates (measured: +16 % per-SM unpack throughput over plain shifts).
__device__ __forceinline__ uint32_t mul_lo_u32(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.lo.u32 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t mul_hi_u32(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.hi.u32 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// Nibble pairs (0,4), (1,5), (2,6), (3,7) of w as fp16x2 offset integers:
// 64 + u (unsigned) or 72 + s (signed two's complement nibble).  Each pair
// is moved to bits 4-7 / 20-23 (w * 16, w, w / 16, w / 256) and merged into
// the mantissa of 64.0 by one LOP3.
template <bool SIGNED>
__device__ __forceinline__ void unpack_offset64(uint32_t w, uint32_t (&e)[4]) {
    constexpr uint32_t kMask = 0x00F000F0u;
    constexpr uint32_t kMagic = SIGNED ? 0x54805480u : 0x54005400u;
    constexpr int kLut = SIGNED ? 0x6A : 0xEA;     // (a & b) ^ c  /  (a & b) | c
    e[0] = lop3<kLut>(mul_lo_u32(w, 16u), kMask, kMagic);
    e[1] = lop3<kLut>(w, kMask, kMagic);
    e[2] = lop3<kLut>(mul_hi_u32(w, 1u << 28), kMask, kMagic);
    e[3] = lop3<kLut>(mul_hi_u32(w, 1u << 24), kMask, kMagic);
}

// Word-row offset (0..15) of lane column c in row step j of a warp's 16 rows;
// with the 64-byte swizzle this makes every quarter-warp read hit 8 distinct
// bank groups (a row step is 4 rows read by the 4 lane columns).
__device__ __forceinline__ int row_of(int j, int c) { return (c & 1) + 4 * (c >> 1) + 2 * (j & 1) + 8 * (j >> 1); }

struct CtaPlan {
    int t0;         // first tile
    int n4;         // groups of four tiles (wide)
    int rem;        // tiles after them (0..3): 2 or 3 -> one narrow group of 2; odd -> one lone tile
    int ng, total;  // groups, stages
};

// A CTA's n tiles are groups of four ("wide": 2 warp columns of 32 columns,
// rows_wide rows per stage), then for a remainder of 2 or 3 one "narrow" group
// of two (1 warp column, rows_narrow rows), then for an odd remainder one lone
// tile.  For M <= 4 a lone tile is a "split" group: the lanes that would read
// the second box of a narrow group read the second row half of the same tile
// instead, so a stage covers rows_split = 2 rows_narrow rows and no lane
// idles.  An MMA has one K range for all its rows, so the halves are kept
// apart in the batch dimension: B column n = 2 m + h carries batch row m over
// row half h (h = n & 1 = bb of the lane that supplies it), and MMA row r --
// weights of half bb(r) -- keeps only the products with columns of its own
// half, elements (e & 1) == bb.  Every kind then moves the same
// 512-word-per-warp stage, so a CTA's stage count is proportional to its tiles
// (a wide group of 3 tiles idled a quarter of the lanes, a lone narrow tile
// half of them).  For M > 4 a lone tile is a narrow group of one.
// First tile of CTA b.  With at least two tiles a CTA, the T mod G tiles left
// over by the even share go one each to the first CTAs: those are dispatched
// first and start first, as the previous kernel's CTAs leave their SMs
// (measured on the decode step: 4096 x 14336 13.1 -> 12.0 us a launch).
// Below two tiles a CTA the shares are spread evenly (b T / G): there the
// extra-first order lost (4096 x 4096: 5.3 -> 5.4-5.8 us).
// T tiles over G CTAs (of one projection).
__device__ __forceinline__ int first_tile(int T, int G, uint32_t b) {
    const int base = T / G;
    if (base >= 2) return (int)b * base + min((int)b, T - base * G);
    return (int)(b * (uint32_t)T / (uint32_t)G);         // b * T < 2^32 (checked on the host)
}

// Tiles and stages of CTA b of the G that share the T tiles of a projection.
__device__ __forceinline__ CtaPlan cta_plan(const DecodeParams& p, int T, int G, uint32_t b) {
    CtaPlan q;
    q.t0 = first_tile(T, G, b);
    const int t1 = first_tile(T, G, b + 1);
    const int n = t1 - q.t0;
    q.n4 = n >> 2;
    q.rem = n & 3;
    q.ng = q.n4 + (q.rem >= 2 ? 1 : 0) + (q.rem & 1);
    q.total = q.n4 * p.s_wide + (q.rem >= 2 ? p.s_narrow : 0) + ((q.rem & 1) ? (p.split ? p.s_split : p.s_narrow) : 0);
    return q;
}

enum GroupKind { kWide = 0, kNarrow = 1, kSplit = 2 };

struct GroupInfo {
    int kind, nt, tile0, nst, stage0;
};

__device__ __forceinline__ GroupInfo group_info(const DecodeParams& p, const CtaPlan& q, int g) {
    GroupInfo gi;
    if (g < q.n4) {
        gi.kind = kWide; gi.nt = 4; gi.tile0 = q.t0 + 4 * g; gi.nst = p.s_wide; gi.stage0 = g * p.s_wide;
        return gi;
    }
    gi.tile0 = q.t0 + 4 * q.n4;
    gi.stage0 = q.n4 * p.s_wide;
    if (q.rem >= 2 && g == q.n4) {
        gi.kind = kNarrow; gi.nt = 2; gi.nst = p.s_narrow;
        return gi;
    }
    if (q.rem >= 2) {           // the lone tile after a narrow group
        gi.tile0 += 2;
        gi.stage0 += p.s_narrow;
    }
    gi.nt = 1;
    gi.kind = p.split ? kSplit : kNarrow;
    gi.nst = p.split ? p.s_split : p.s_narrow;
    return gi;
}

// Issue ring stage i (global stage index within this CTA) into `slot`.
template <int MT, bool HAS_ZP>
__device__ __forceinline__ void issue_stage(const DecodeParams& p, const CtaPlan& q, const ProjMaps& maps,
                                            uint8_t* ring, uint64_t* full, int i, int slot) {
    using S = Shape<MT>;
    int g = (i < q.n4 * p.s_wide) ? i / p.s_wide : q.n4;
    GroupInfo gi = group_info(p, q, g);
    if (i >= gi.stage0 + gi.nst) gi = group_info(p, q, ++g);     // past the narrow group: the lone tile
    const int ks = i - gi.stage0;
    uint8_t* base = ring + (size_t)slot * p.slot_bytes;
    uint8_t* sbase = base + S::kWeightBytes;
    if (gi.kind == kSplit) {
        // two boxes of rows_narrow rows: the two row halves of one tile
        const int row0 = ks * S::kRowsSplit;
        const uint32_t sbox = (uint32_t)p.sbr_split * 32;
        mbar_arrive_expect_tx(&full[slot], (uint32_t)(2 * S::kRowsNarrow * 64) + sbox * (HAS_ZP ? 2 : 1));
        tma_load_2d(base, &maps.w_narrow, kBoxCols * gi.tile0, row0, &full[slot]);
        tma_load_2d(base + S::kRowsNarrow * 64, &maps.w_narrow, kBoxCols * gi.tile0, row0 + S::kRowsNarrow, &full[slot]);
        const int sr = (p.gw_shift >= 0) ? (row0 >> p.gw_shift) : row0 / p.gw;
        tma_load_2d(sbase, &maps.s_split, kBoxCols * gi.tile0, sr, &full[slot]);
        if constexpr (HAS_ZP) tma_load_2d(sbase + p.s_bytes, &maps.z_split, kBoxCols * gi.tile0, sr, &full[slot]);
        return;
    }
    const bool wide = gi.kind == kWide;
    const int rows = wide ? S::kRowsWide : S::kRowsNarrow;
    const int row0 = ks * rows;
    const uint32_t sbox = wide ? (uint32_t)p.sbr_wide * 128 : (uint32_t)p.sbr_narrow * 64;
    mbar_arrive_expect_tx(&full[slot], (uint32_t)(gi.nt * rows * 64) + sbox * (HAS_ZP ? 2 : 1));
    const CUtensorMap* tw = wide ? &maps.w_wide : &maps.w_narrow;
    for (int bx = 0; bx < gi.nt; ++bx)
        tma_load_2d(base + bx * rows * 64, tw, kBoxCols * (gi.tile0 + bx), row0, &full[slot]);
    const int sr = (p.gw_shift >= 0) ? (row0 >> p.gw_shift) : row0 / p.gw;
    tma_load_2d(sbase, wide ? &maps.s_wide : &maps.s_narrow, kBoxCols * gi.tile0, sr, &full[slot]);
    if constexpr (HAS_ZP)
        tma_load_2d(sbase + p.s_bytes, wide ? &maps.z_wide : &maps.z_narrow, kBoxCols * gi.tile0, sr, &full[slot]);
}

// acc += s * (dg + o * sum a) for the two 16-column sub-tiles of this lane,
// o = -(offset + z).  s / z: the lane's four columns 4L..4L+3.  The sums are
// those of the lane's batch rows 2c, 2c+1 -- or, in a split group (SPLIT), of
// its one batch row c over its row half, the same value for both.
template <int MT, bool SIGNED, bool HAS_ZP, bool SPLIT>
__device__ __forceinline__ void flush(float (&acc)[MT][2][4], const float (&dg)[MT][2][4], uint32_t saddr,
                                      uint32_t zaddr, uint32_t sum_addr) {
    constexpr float kOff = SIGNED ? 72.f : 64.f;
    const uint2 sv = lds64(saddr);
    float s[4] = {h_to_f((uint16_t)(sv.x & 0xFFFF)), h_to_f((uint16_t)(sv.x >> 16)),
                  h_to_f((uint16_t)(sv.y & 0xFFFF)), h_to_f((uint16_t)(sv.y >> 16))};
    float o[4] = {-kOff, -kOff, -kOff, -kOff};
    if constexpr (HAS_ZP) {
        const uint2 zv = lds64(zaddr);
        o[0] = -(kOff + h_to_f((uint16_t)(zv.x & 0xFFFF)));
        o[1] = -(kOff + h_to_f((uint16_t)(zv.x >> 16)));
        o[2] = -(kOff + h_to_f((uint16_t)(zv.y & 0xFFFF)));
        o[3] = -(kOff + h_to_f((uint16_t)(zv.y >> 16)));
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
        float sa[2];
        if constexpr (SPLIT) {
            sa[0] = sa[1] = lds32f(sum_addr + 32 * mt);
        } else {
            const uint2 sv2 = lds64(sum_addr + 32 * mt);
            sa[0] = __uint_as_float(sv2.x);
            sa[1] = __uint_as_float(sv2.y);
        }
#pragma unroll
        for (int X = 0; X < 2; ++X)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int k = 2 * X + (e >> 1);
                acc[mt][X][e] = fmaf(s[k], fmaf(o[k], sa[e & 1], dg[mt][X][e]), acc[mt][X][e]);
            }
    }
}

// Barrier operations by 32-bit shared-memory address (the math warps keep
// addresses, not 64-bit generic pointers, live across the stage loop).
__device__ __forceinline__ bool try_wait_a(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ bool wait_bounded_a(uint32_t bar, uint32_t parity) {
    if (try_wait_a(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        if (try_wait_a(bar, parity)) return true;
        if (global_timer_ns() - t0 > kWaitLimitNs) return false;
    }
}

__device__ __forceinline__ void arrive_a(uint32_t bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* addr, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(addr), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* addr) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(addr) : "memory");
    return v;
}

// State the math warps carry from one tile group to the next.
struct MathCtx {
    uint32_t ring_a, act_a, sums_a, pitch16;
    uint32_t full_a, empty_a;   // barrier arrays (8 bytes per slot)
    float* red;
    volatile int* sflag;
    int warp, lane, r, c, bb, L;
    int slot;
    uint32_t phase;
    uint32_t epoch;         // fused all-gather: this call's epoch (0 on one GPU)
    uint16_t* C;            // the CTA's projection: output and its columns
    int N;
    int col_off;            // fused all-gather: its first column in the group buffer
    bool aborted;
    int group;          // groups done (selects the reduction buffer)
};

// This lane's shared-memory offsets in a stage of a KIND group.  Loads are
// unconditional (a guard around inline asm becomes a branch that splits the
// stage into small scheduling regions): a lane whose box lies past the
// group's last tile reads another box of the slot, and a lane past the last
// batch row reads row M-1; both only feed MMA rows / columns never stored.
template <int MT>
struct LaneOffsets {
    uint32_t woff[4];       // packed words, row step j
    uint32_t aoff[MT][4];   // activation records, row step j (plus the stage's row0 * 16)
    uint32_t soff[2];       // scales of flush half h
    int lane_row;           // first word row of this lane's rows in a stage
};

template <int MT, int KIND>
__device__ __forceinline__ LaneOffsets<MT> setup_lane(const DecodeParams& p, const MathCtx& x) {
    using S = Shape<MT>;
    constexpr int nwc = (KIND == kWide) ? 2 : 1;                 // warp columns (32 columns each)
    constexpr int rbs = S::kWarps / nwc;                          // 16-row blocks per box
    constexpr int box_rows = (KIND == kWide) ? S::kRowsWide : S::kRowsNarrow;
    constexpr int rows = (KIND == kSplit) ? S::kRowsSplit : box_rows;
    constexpr int srow_bytes = (KIND == kWide) ? 128 : (KIND == kNarrow ? 64 : 32);
    LaneOffsets<MT> lo;
    const int wc = (nwc == 2) ? x.warp / rbs : 0;
    const int rb = x.warp - wc * rbs;
    const int box = 2 * wc + x.bb;                                // a split group's box bb is row half bb
    lo.lane_row = 16 * rb + ((KIND == kSplit) ? x.bb * S::kRowsNarrow : 0);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int row = 16 * rb + row_of(j, x.c);                 // row within the box
        lo.woff[j] = (uint32_t)(box * box_rows * 64 + row * 64) + (uint32_t)((x.L ^ ((row >> 1) & 3)) << 4);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            const int m = (KIND == kSplit) ? min(x.r >> 1, p.M - 1) : min(x.r + 8 * mt, p.M - 1);
            lo.aoff[mt][j] = x.act_a + (uint32_t)m * x.pitch16 + (uint32_t)(lo.lane_row + row_of(j, x.c)) * 16;
        }
    }
    // scale row of this lane's flush blocks (rows lane_row + 8h of the stage); a
    // scale box row holds the group's 64 (wide), 32 (narrow) or 16 (split) columns
    const int scol = (KIND == kSplit) ? 4 * x.L : 16 * box + 4 * x.L;
    const bool per_row = p.gw_shift >= 0 && p.gw < rows;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int srow = per_row ? ((lo.lane_row + 8 * h) >> p.gw_shift) : 0;
        lo.soff[h] = (uint32_t)(S::kWeightBytes + srow * srow_bytes + scol * 2);
    }
    return lo;
}

template <int MT>
__device__ __forceinline__ LaneOffsets<MT> setup_any(int kind, const DecodeParams& p, const MathCtx& x) {
    if (kind == kWide) return setup_lane<MT, kWide>(p, x);
    if (MT == 1 && kind == kSplit) return setup_lane<MT, kSplit>(p, x);
    return setup_lane<MT, kNarrow>(p, x);
}

// The math of one ring stage for this warp: its 16 rows x 32 columns of the
// stage in slot address `st`, flushed into acc.
template <int MT, bool SIGNED, bool HAS_ZP, bool FB8, int KIND>
__device__ __forceinline__ void stage_math(const DecodeParams& p, const LaneOffsets<MT>& lo, float (&acc)[MT][2][4],
                                           uint32_t st, int row0, uint32_t sum_base) {
    constexpr bool kSplitGroup = KIND == kSplit;
    const uint32_t zdelta = (uint32_t)p.s_bytes;
    const uint32_t arow = (uint32_t)row0 * 16;
    float dg[MT][2][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint4 wv = lds128(st + lo.woff[j]);
        uint4 av[MT];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) av[mt] = lds128(lo.aoff[mt][j] + arow);
        uint32_t e0[4], e1[4], e2[4], e3[4];
        unpack_offset64<SIGNED>(wv.x, e0);   // column 4L     (sub-tile 0, MMA row r)
        unpack_offset64<SIGNED>(wv.y, e1);   // column 4L + 1 (sub-tile 0, MMA row r + 8)
        unpack_offset64<SIGNED>(wv.z, e2);   // column 4L + 2 (sub-tile 1, MMA row r)
        unpack_offset64<SIGNED>(wv.w, e3);   // column 4L + 3 (sub-tile 1, MMA row r + 8)
        const bool first = (j == 0) || (j == 2 && FB8);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            if (first) {
                mma_16816_zero(dg[mt][0], e0[0], e1[0], e0[1], e1[1], av[mt].x, av[mt].y);
                mma_16816_zero(dg[mt][1], e2[0], e3[0], e2[1], e3[1], av[mt].x, av[mt].y);
            } else {
                mma_16816(dg[mt][0], e0[0], e1[0], e0[1], e1[1], av[mt].x, av[mt].y);
                mma_16816(dg[mt][1], e2[0], e3[0], e2[1], e3[1], av[mt].x, av[mt].y);
            }
            mma_16816(dg[mt][0], e0[2], e1[2], e0[3], e1[3], av[mt].z, av[mt].w);
            mma_16816(dg[mt][1], e2[2], e3[2], e2[3], e3[3], av[mt].z, av[mt].w);
        }
        if (j == 1 && FB8) {
            const uint32_t b8 = (uint32_t)((row0 + lo.lane_row) >> 3);
            flush<MT, SIGNED, HAS_ZP, kSplitGroup>(acc, dg, st + lo.soff[0], st + lo.soff[0] + zdelta,
                                                   sum_base + b8 * (32 * MT));
        }
    }
    if (FB8) {
        const uint32_t b8 = (uint32_t)((row0 + lo.lane_row) >> 3) + 1;
        flush<MT, SIGNED, HAS_ZP, kSplitGroup>(acc, dg, st + lo.soff[1], st + lo.soff[1] + zdelta,
                                               sum_base + b8 * (32 * MT));
    } else {
        const uint32_t b16 = (uint32_t)((row0 + lo.lane_row) >> 4);
        flush<MT, SIGNED, HAS_ZP, kSplitGroup>(acc, dg, st + lo.soff[0], st + lo.soff[0] + zdelta,
                                               sum_base + b16 * (32 * MT));
    }
}

// The math of two ring stages for this warp, interleaved row step by row
// step: the two stages' loads, unpacking and MMAs are independent chains, so
// one warp has twice the work in flight between two barrier waits.
template <int MT, bool SIGNED, bool HAS_ZP, bool FB8, int KIND>
__device__ __forceinline__ void stage_math2(const DecodeParams& p, const LaneOffsets<MT>& lo, float (&acc)[MT][2][4],
                                            uint32_t st0, uint32_t st1, int row0, int row1, uint32_t sum_base) {
    constexpr bool kSplitGroup = KIND == kSplit;
    const uint32_t zdelta = (uint32_t)p.s_bytes;
    const uint32_t st[2] = {st0, st1};
    const int r0[2] = {row0, row1};
    float dg[2][MT][2][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint4 wv[2], av[2][MT];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            wv[h] = lds128(st[h] + lo.woff[j]);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) av[h][mt] = lds128(lo.aoff[mt][j] + (uint32_t)r0[h] * 16);
        }
        const bool first = (j == 0) || (j == 2 && FB8);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            uint32_t e0[4], e1[4], e2[4], e3[4];
            unpack_offset64<SIGNED>(wv[h].x, e0);
            unpack_offset64<SIGNED>(wv[h].y, e1);
            unpack_offset64<SIGNED>(wv[h].z, e2);
            unpack_offset64<SIGNED>(wv[h].w, e3);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                if (first) {
                    mma_16816_zero(dg[h][mt][0], e0[0], e1[0], e0[1], e1[1], av[h][mt].x, av[h][mt].y);
                    mma_16816_zero(dg[h][mt][1], e2[0], e3[0], e2[1], e3[1], av[h][mt].x, av[h][mt].y);
                } else {
                    mma_16816(dg[h][mt][0], e0[0], e1[0], e0[1], e1[1], av[h][mt].x, av[h][mt].y);
                    mma_16816(dg[h][mt][1], e2[0], e3[0], e2[1], e3[1], av[h][mt].x, av[h][mt].y);
                }
                mma_16816(dg[h][mt][0], e0[2], e1[2], e0[3], e1[3], av[h][mt].z, av[h][mt].w);
                mma_16816(dg[h][mt][1], e2[2], e3[2], e2[3], e3[3], av[h][mt].z, av[h][mt].w);
            }
        }
        if (j == 1 && FB8) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t b8 = (uint32_t)((r0[h] + lo.lane_row) >> 3);
                flush<MT, SIGNED, HAS_ZP, kSplitGroup>(acc, dg[h], st[h] + lo.soff[0], st[h] + lo.soff[0] + zdelta,
                                                       sum_base + b8 * (32 * MT));
            }
        }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        if (FB8) {
            const uint32_t b8 = (uint32_t)((r0[h] + lo.lane_row) >> 3) + 1;
            flush<MT, SIGNED, HAS_ZP, kSplitGroup>(acc, dg[h], st[h] + lo.soff[1], st[h] + lo.soff[1] + zdelta,
                                                   sum_base + b8 * (32 * MT));
        } else {
            const uint32_t b16 = (uint32_t)((r0[h] + lo.lane_row) >> 4);
            flush<MT, SIGNED, HAS_ZP, kSplitGroup>(acc, dg[h], st[h] + lo.soff[0], st[h] + lo.soff[0] + zdelta,
                                                   sum_base + b16 * (32 * MT));
        }
    }
}

// Bounded wait for the stage in the current slot; an abort (timeout) is
// recorded once and every later stage is skipped.
__device__ __forceinline__ void wait_stage(MathCtx& x, uint32_t slot, uint32_t phase) {
    if (!x.aborted && !wait_bounded_a(x.full_a + 8u * slot, phase)) {
        x.aborted = true;
        x.sflag[0] = 1;
        atomicOr(&g_decode_error, kErrTimeout);
    }
}

__device__ __forceinline__ void next_slot(const DecodeParams& p, uint32_t& slot, uint32_t& phase) {
    if (++slot == (uint32_t)p.stages) {
        slot = 0;
        phase ^= 1u;
    }
}

// Stream one tile group's stages through the ring and store its outputs.
// Stages are taken two at a time: both waits, then both stages' math as one
// block the compiler can interleave (loads and unpacking of the second under
// the MMAs and flush of the first), then both releases.  A stage at a time,
// every warp stalled on the same exposed latencies at each stage boundary
// (measured: 1485 against 965 cycles per stage for the same math unfenced).
// Holding two slots is safe: the ring has at least two, and a stage's slot was
// released by this warp before (ks >= stages) or never used.
template <int MT, bool SIGNED, bool HAS_ZP, bool FB8, int KIND>
__device__ __forceinline__ void run_group(const DecodeParams& p, const GroupInfo& gi, const LaneOffsets<MT>& lo,
                                          MathCtx& x) {
    using S = Shape<MT>;
    constexpr int kWarps = S::kWarps;
    constexpr int kMathThreads = 32 * kWarps;
    constexpr int nwc = (KIND == kWide) ? 2 : 1;
    constexpr int rbs = kWarps / nwc;
    constexpr int rows = (KIND == kSplit) ? S::kRowsSplit : ((KIND == kWide) ? S::kRowsWide : S::kRowsNarrow);
    constexpr bool kSplitGroup = KIND == kSplit;
    const uint32_t sum_base = kSplitGroup ? x.sums_a + (uint32_t)x.c * 4 : x.sums_a + (uint32_t)(2 * x.c) * 4;

    float acc[MT][2][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int X = 0; X < 2; ++X)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[mt][X][e] = 0.f;

    uint32_t slot = (uint32_t)x.slot, phase = x.phase;
    int ks = 0;
    for (; ks + 1 < gi.nst; ks += 2) {
        uint32_t slot1 = slot, phase1 = phase;
        next_slot(p, slot1, phase1);
        wait_stage(x, slot, phase);
        wait_stage(x, slot1, phase1);
        if (!x.aborted)
            stage_math2<MT, SIGNED, HAS_ZP, FB8, KIND>(p, lo, acc, x.ring_a + slot * (uint32_t)p.slot_bytes,
                                                      x.ring_a + slot1 * (uint32_t)p.slot_bytes, ks * rows,
                                                      (ks + 1) * rows, sum_base);
        // every lane's reads of both slots are complete (their results fed
        // the MMAs above): release them to the producer
        __syncwarp();
        if (x.lane == 0) {
            arrive_a(x.empty_a + 8u * slot);
            arrive_a(x.empty_a + 8u * slot1);
        }
        slot = slot1;
        phase = phase1;
        next_slot(p, slot, phase);
    }
    if (ks < gi.nst) {
        wait_stage(x, slot, phase);
        if (!x.aborted)
            stage_math<MT, SIGNED, HAS_ZP, FB8, KIND>(p, lo, acc, x.ring_a + slot * (uint32_t)p.slot_bytes, ks * rows,
                                                     sum_base);
        __syncwarp();
        if (x.lane == 0) arrive_a(x.empty_a + 8u * slot);
        next_slot(p, slot, phase);
    }
    x.slot = (int)slot;
    x.phase = phase;

    // ---- group done: sum the row blocks of each warp column in a fixed order.
    // A column's M partial sums sit rs = M | 1 floats apart: with an odd
    // stride, the lanes of a warp (one column each on the read side, 8 columns
    // x 4 batch rows on the write side) fall in distinct banks or at most two
    // to a bank, where a stride of 16 put 16 lanes on one bank.
    const int M = p.M;
    const int rs = M | 1;
    // two reduction buffers, alternating by group: the next group writes the
    // other one, so the warps that sum this group's columns need no barrier
    // after them (the group after next waits at its own barrier, which every
    // warp reaches only after finishing this group's sums)
    float* red = x.red + (x.group & 1) * (p.red_floats >> 1);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int X = 0; X < 2; ++X)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int col = 16 * x.bb + 4 * x.L + 2 * X + (e >> 1);
                if (kSplitGroup) {       // batch row c, own row half only
                    if ((e & 1) == x.bb && x.c < M) red[(x.warp * 32 + col) * rs + x.c] = acc[mt][X][e];
                } else {
                    const int m = 8 * mt + 2 * x.c + (e & 1);
                    if (m < M) red[(x.warp * 32 + col) * rs + m] = acc[mt][X][e];
                }
            }
    named_barrier(1, kMathThreads);
    const int col_base = kBoxCols * gi.tile0;
    int ncols = kBoxCols * gi.nt;
    if (col_base + ncols > x.N) ncols = x.N - col_base;
    for (int pair = x.warp; pair < nwc * M; pair += kWarps) {
        const int w = pair / M, m = pair - w * M;
        const int col = 32 * w + x.lane;
        uint32_t hv = 0;
        if (col < ncols) {
            float v = 0.f;
            for (int k = 0; k < rbs; ++k) v += red[((w * rbs + k) * 32 + x.lane) * rs + m];
            if (kSplitGroup)     // the second row half sits in columns 16..31 of each row block
                for (int k = 0; k < rbs; ++k) v += red[(k * 32 + x.lane + kBoxCols) * rs + m];
            const uint16_t h = __half_as_ushort(__float2half_rn(v));
            if (p.world == 1) x.C[(size_t)m * x.N + col_base + col] = h;
            hv = h;
        }
        if (p.world > 1) {
            // Even lanes pair their column with the next one (ncols is even,
            // and every lane of the warp runs this iteration) and store
            // {col, col+1, epoch} as one word into every rank's receive buffer
            // (peer memory over NVLink): a reader that sees the epoch sees
            // the data, so no fence or flag is needed.
            const uint32_t hi = __shfl_down_sync(0xffffffffu, hv, 1);
            if (col < ncols && (x.lane & 1) == 0) {
                const unsigned long long word = ((unsigned long long)x.epoch << 32) | (hv | (hi << 16));
                const size_t o = ((size_t)(x.epoch & 1u) * M + m) * (size_t)(p.n_total >> 1) +
                                 (size_t)((x.col_off + col_base + col) >> 1);
                for (int g = 0; g < p.world; ++g) st_relaxed_sys_u64(p.recv[g] + o, word);
            }
        }
    }
    ++x.group;
}

// End of a CTA of the launch that closes a fused all-gather group (every
// thread).  The CTA's slice of the group's words in this rank's receive
// buffer is polled until each carries this call's epoch (bounded), and the
// column pairs go to the local output.  Every CTA of the launch is resident
// at once (the grid is at most one CTA per SM), so a CTA waiting here never
// keeps the CTAs that produce its words from running.  The last CTA to finish
// advances the epoch: every CTA of the launch read it before arriving, and
// the next call reads it only after this launch has ended.
__device__ __forceinline__ void gather_complete(const DecodeParams& p) {
    const uint32_t epoch = *reinterpret_cast<volatile const unsigned*>(p.counter + 1) + 1u;
    const int words = p.M * (p.n_total >> 1);
    const int per = (words + gridDim.x - 1) / gridDim.x;
    const int lo = blockIdx.x * per;
    const int hi = lo + per < words ? lo + per : words;
    const unsigned long long* src = p.recv[p.rank] + (size_t)(epoch & 1u) * words;
    constexpr int kBatch = 4;
    const uint64_t t0 = global_timer_ns();
    bool ok = true;
    for (int base = lo + (int)threadIdx.x; ok && base < hi; base += kBatch * blockDim.x) {
        unsigned long long v[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const int i = base + u * (int)blockDim.x;
            v[u] = i < hi ? ld_relaxed_sys_u64(src + i) : ((unsigned long long)epoch << 32);
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const int i = base + u * (int)blockDim.x;
            while (ok && (uint32_t)(v[u] >> 32) != epoch) {
                if (global_timer_ns() - t0 > kWaitLimitNs) {
                    atomicOr(&g_decode_error, kErrTimeout);
                    ok = false;
                } else {
                    v[u] = ld_relaxed_sys_u64(src + i);
                }
            }
            if (ok && i < hi) p.gout[i] = (uint32_t)v[u];
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();     // this CTA's read of the epoch is done before it arrives
        if (atomicAdd(p.counter, 1u) == gridDim.x - 1) {
            p.counter[0] = 0u;
            p.counter[1] = epoch;
        }
    }
}

// One CTA per SM (its ring takes the SM's shared memory), so the register
// budget is that of one CTA.  NP: the projections a launch can hold (1, or
// kMaxProj for a grouped launch); each CTA works on one of them.
template <int MT, bool SIGNED, bool HAS_ZP, bool FB8, int NP>
__global__ void __launch_bounds__(Shape<MT>::kThreads, 1)
gemv_w4_decode_kernel(const __grid_constant__ DecodeMaps<NP> maps, const DecodeParams p) {
    using S = Shape<MT>;
    constexpr int kWarps = S::kWarps;
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned ring (pointer arithmetic on smem_raw keeps the
    // compiler aware that every access below is to shared memory)
    uint8_t* ring = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    uint8_t* act = ring + (size_t)p.stages * p.slot_bytes;
    float* sums = reinterpret_cast<float*>(act + p.act_bytes);
    float* red = sums + p.sum_floats;
    uint64_t* full = reinterpret_cast<uint64_t*>(red + p.red_floats);
    uint64_t* empty = full + kMaxStages;       // one arrival per math warp
    uint64_t* prep_done = empty + kMaxStages;  // the activations are in place
    volatile int* sflag = reinterpret_cast<volatile int*>(prep_done + 1);   // [0] abort, [1] stages issued

    pdl_launch_dependents();
    int j = 0;          // this CTA's projection
#pragma unroll
    for (int i = 1; i < NP; ++i)
        if (i < p.nproj && (int)blockIdx.x >= p.proj_g0[i]) j = i;
    const ProjMaps& pm = maps.proj[j];
    const CtaPlan q = cta_plan(p, p.proj_T[j], p.proj_g0[j + 1] - p.proj_g0[j], blockIdx.x - (uint32_t)p.proj_g0[j]);
    const int tid = threadIdx.x;
    constexpr int kMathThreads = 32 * kWarps;
    if (tid == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kWarps);
        }
        mbar_init(prep_done, 1);
        sflag[0] = 0;
        sflag[1] = 0;
        fence_barrier_init();
    }
    __syncthreads();

    if (tid >= kMathThreads) {
        // ---------------- producer warp: every TMA copy of the ring
        if (tid == kMathThreads) {
            prefetch_tmap(&pm.w_wide);
            prefetch_tmap(&pm.w_narrow);
            prefetch_tmap(&pm.s_wide);
            prefetch_tmap(&pm.s_narrow);
            prefetch_tmap(&pm.s_split);
            if constexpr (HAS_ZP) {
                prefetch_tmap(&pm.z_wide);
                prefetch_tmap(&pm.z_narrow);
                prefetch_tmap(&pm.z_split);
            }
            // weights, scales and zero points are never written by a kernel of
            // this library, so they may be fetched before the previous kernel ends
            const int early = q.total < p.early ? q.total : p.early;
            for (int s = 0; s < early; ++s) issue_stage<MT, HAS_ZP>(p, q, pm, ring, full, s, s);
            sflag[1] = early;
            // The rest of the ring only once the activations are in: their
            // loads are on the critical path and should not queue behind this
            // SM's weight stream.
            bool ok = mbar_wait_bounded(prep_done, 0, kWaitLimitNs);
            for (int i = early; ok && i < q.total; ++i) {
                const int slot = i % p.stages;
                if (i >= p.stages && !mbar_wait_bounded(&empty[slot], (uint32_t)(((i / p.stages) & 1) ^ 1), kWaitLimitNs))
                    ok = false;
                if (!ok || sflag[0]) break;
                fence_proxy_async_smem();     // the math warps' reads of the slot before the copy overwrites it
                issue_stage<MT, HAS_ZP>(p, q, pm, ring, full, i, slot);
                sflag[1] = i + 1;
            }
            if (!ok) {
                sflag[0] = 1;
                atomicOr(&g_decode_error, kErrTimeout);
            }
        }
    } else {
    // ---- per-lane constants and the offsets of the first tile group: none of
    // it depends on the previous kernel, so the math warps compute it while
    // that kernel drains instead of after the activations are in.
    MathCtx x;
    x.warp = tid >> 5;
    x.lane = tid & 31;
    x.r = x.lane >> 2;
    x.c = x.lane & 3;
    x.bb = x.r & 1;                           // which of the warp's two boxes (row half in a split group)
    x.L = (x.r >> 1) ^ (x.r & 1);             // 16-byte chunk (4 columns) of that box
    x.ring_a = smem_addr(ring);
    x.act_a = smem_addr(act);
    x.sums_a = smem_addr(sums);
    x.pitch16 = (uint32_t)(p.KWp + 2) * 16;
    x.red = red;
    x.full_a = smem_addr(full);
    x.empty_a = smem_addr(empty);
    x.sflag = sflag;
    x.slot = 0;
    x.phase = 0;
    x.epoch = 0;
    x.C = p.proj_C[j];
    x.N = p.proj_N[j];
    x.col_off = p.proj_coloff[j];
    x.aborted = false;
    x.group = 0;
    GroupInfo gi = group_info(p, q, 0);
    LaneOffsets<MT> lo = setup_any<MT>(gi.kind, p, x);

    pdl_wait_prior_grid();     // A and C may belong to the previous kernel
    if (p.world > 1) x.epoch = *reinterpret_cast<volatile const unsigned*>(p.counter + 1) + 1u;

    // ---- resident activations: permuted records + flush-block sums.  Every
    // thread issues kPrep independent loads before using any, so the prologue
    // costs one L2 round trip per batch, not one per record.
    {
        constexpr int kPrep = 4;
        const int MB = 8 * MT;
        const int items = p.M * p.KWp;      // a multiple of 128: every test below is uniform per warp
        const uint32_t pitch = (uint32_t)(p.KWp + 2);
        for (int base = 0; base < items; base += kMathThreads * kPrep) {
            uint4 v[kPrep];
#pragma unroll
            for (int k = 0; k < kPrep; ++k) {
                const int it = base + k * kMathThreads + tid;
                const int m = (int)fdiv((uint32_t)it, p.kwdiv);
                const int kw = it - m * p.KWp;
                v[k] = make_uint4(0, 0, 0, 0);
                if (it < items && kw < p.KW)
                    v[k] = __ldcg(reinterpret_cast<const uint4*>(p.A + (size_t)m * p.K + 8 * (size_t)kw));
            }
#pragma unroll
            for (int k = 0; k < kPrep; ++k) {
                const int it = base + k * kMathThreads + tid;
                if (it >= items) continue;      // uniform per warp (the shuffles below need all 32 lanes)
                const int m = (int)fdiv((uint32_t)it, p.kwdiv);
                const int kw = it - m * p.KWp;
                uint4 rec;
                rec.x = prmt(v[k].x, v[k].z, 0x5410);
                rec.y = prmt(v[k].x, v[k].z, 0x7632);
                rec.z = prmt(v[k].y, v[k].w, 0x5410);
                rec.w = prmt(v[k].y, v[k].w, 0x7632);
                *reinterpret_cast<uint4*>(act + ((size_t)m * pitch + kw) * 16) = rec;
                const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&v[k].x));
                const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&v[k].y));
                const float2 f2 = __half22float2(*reinterpret_cast<const __half2*>(&v[k].z));
                const float2 f3 = __half22float2(*reinterpret_cast<const __half2*>(&v[k].w));
                float s = ((f0.x + f0.y) + (f1.x + f1.y)) + ((f2.x + f2.y) + (f3.x + f3.y));
                s += __shfl_xor_sync(0xffffffffu, s, 1);
                s += __shfl_xor_sync(0xffffffffu, s, 2);
                s += __shfl_xor_sync(0xffffffffu, s, 4);
                if (p.fb == 16) s += __shfl_xor_sync(0xffffffffu, s, 8);
                if ((kw & (p.fb - 1)) == 0) sums[(kw / p.fb) * MB + m] = s;
            }
        }
        for (int idx = tid; idx < p.sum_floats; idx += kMathThreads)
            if ((idx & (MB - 1)) >= p.M) sums[idx] = 0.f;
    }
    named_barrier(1, kMathThreads);
    if (tid == 0) mbar_arrive(prep_done);

    for (int g = 0; g < q.ng; ++g) {
        if (g > 0) {
            gi = group_info(p, q, g);
            lo = setup_any<MT>(gi.kind, p, x);
        }
        if (gi.kind == kWide) {
            run_group<MT, SIGNED, HAS_ZP, FB8, kWide>(p, gi, lo, x);
        } else if (MT == 1 && gi.kind == kSplit) {
            run_group<MT, SIGNED, HAS_ZP, FB8, kSplit>(p, gi, lo, x);
        } else {
            run_group<MT, SIGNED, HAS_ZP, FB8, kNarrow>(p, gi, lo, x);
        }
    }
    }   // math warps

    __syncthreads();
    if (sflag[0] && tid == 0) {
        // do not leave while copies may still be landing in this CTA's memory
        const int issued = sflag[1];
        for (int j = (issued > p.stages ? issued - p.stages : 0); j < issued; ++j)
            mbar_wait_bounded(&full[j % p.stages], (uint32_t)((j / p.stages) & 1), kWaitLimitNs / 4);
    }
    if (p.world > 1 && p.barrier) gather_complete(p);
}

template <int MT, bool SIGNED, bool HAS_ZP, bool FB8, int NP>
int launch(const DecodeMaps<NP>& maps, const DecodeParams& p, size_t smem, cudaStream_t stream) {
    auto kern = gemv_w4_decode_kernel<MT, SIGNED, HAS_ZP, FB8, NP>;
    static SmemLimit limit;     // per instantiation, per device
    const int st = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), (int)smem, &limit);
    if (st != T4B_OK) return st;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.G, 1, 1);
    cfg.blockDim = dim3(Shape<MT>::kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t err = cudaLaunchKernelEx(&cfg, kern, maps, p);
    if (err != cudaSuccess) return record_cuda_error(err);
    return T4B_OK;
}

template <int MT, bool SIGNED, int NP>
int dispatch_zp(bool zp, bool fb8, const DecodeMaps<NP>& maps, const DecodeParams& p, size_t smem,
                cudaStream_t stream) {
    if (zp) return fb8 ? launch<MT, SIGNED, true, true, NP>(maps, p, smem, stream)
                       : launch<MT, SIGNED, true, false, NP>(maps, p, smem, stream);
    return fb8 ? launch<MT, SIGNED, false, true, NP>(maps, p, smem, stream)
               : launch<MT, SIGNED, false, false, NP>(maps, p, smem, stream);
}

template <int NP>
int dispatch(bool is_signed, bool zp, bool fb8, int MT, const DecodeMaps<NP>& maps, const DecodeParams& p,
             size_t smem, cudaStream_t stream) {
    if (MT == 1)
        return is_signed ? dispatch_zp<1, true, NP>(zp, fb8, maps, p, smem, stream)
                         : dispatch_zp<1, false, NP>(zp, fb8, maps, p, smem, stream);
    return is_signed ? dispatch_zp<2, true, NP>(zp, fb8, maps, p, smem, stream)
                     : dispatch_zp<2, false, NP>(zp, fb8, maps, p, smem, stream);
}

// Dynamic shared memory one CTA may use on the current device (cached per device).
size_t smem_budget() {
    static std::atomic<int> cached[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && cached[dev].load(std::memory_order_relaxed) > 0)
        return (size_t)cached[dev].load(std::memory_order_relaxed);
    int optin = 0;
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (dev >= 0 && dev < 64) cached[dev].store(optin, std::memory_order_relaxed);
    return (size_t)optin;
}

}  // namespace

int decode_device_error(cudaStream_t stream, unsigned* out, bool clear) {
    unsigned* word = nullptr;
    cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&word), g_decode_error);
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, word, sizeof(unsigned), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess && clear) e = cudaMemsetAsync(word, 0, sizeof(unsigned), stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    return e == cudaSuccess ? T4B_OK : record_cuda_error(e);
}

// Tensor maps of one projection (box shapes of the plan in p).
static bool make_proj_maps(ProjMaps& m, const void* W, const void* S, const void* Z, int N, int K, int group,
                           int rows_wide, int rows_narrow, const DecodeParams& p) {
    const uint64_t KW = (uint64_t)(K / 8), G = (uint64_t)(K / group), n = (uint64_t)N;
    if (!make_tmap_2d_ex(&m.w_wide, false, W, KW, n, rows_wide, kBoxCols, 64, 128) ||
        !make_tmap_2d_ex(&m.w_narrow, false, W, KW, n, rows_narrow, kBoxCols, 64, 128) ||
        !make_tmap_2d_ex(&m.s_wide, true, S, G, n, p.sbr_wide, 4 * kBoxCols, 0, 0) ||
        !make_tmap_2d_ex(&m.s_narrow, true, S, G, n, p.sbr_narrow, 2 * kBoxCols, 0, 0) ||
        !make_tmap_2d_ex(&m.s_split, true, S, G, n, p.sbr_split, kBoxCols, 0, 0))
        return false;
    if (Z) {
        return make_tmap_2d_ex(&m.z_wide, true, Z, G, n, p.sbr_wide, 4 * kBoxCols, 0, 0) &&
               make_tmap_2d_ex(&m.z_narrow, true, Z, G, n, p.sbr_narrow, 2 * kBoxCols, 0, 0) &&
               make_tmap_2d_ex(&m.z_split, true, Z, G, n, p.sbr_split, kBoxCols, 0, 0);
    }
    m.z_wide = m.s_wide;       // never read
    m.z_narrow = m.s_narrow;
    m.z_split = m.s_split;
    return true;
}

// The decode launch of np projections that read the same A (np = 1 for the
// single ops and the fused gather).  Z is NULL (no zero points) or np
// pointers, all set.  plan_only: run every check and the shared-memory plan,
// launch nothing (no pointer is read; Z only says whether there are zero
// points).  ctas, if given, receives each projection's CTA count.  With a
// fused all-gather, col_offsets gives each projection's first column in the
// group buffer (NULL: gather->col_offset, one projection).
static int decode_impl(bool is_signed, const void* A, int np, const void* const* W, const void* const* S,
                       const void* const* Z, void* const* C, const int* N, int M, int K, int group,
                       const T4BGather* gather, cudaStream_t stream, bool plan_only = false, int* ctas = nullptr,
                       const int* col_offsets = nullptr) {
    if (np < 1 || np > kMaxProj || (gather && np != 1 && !col_offsets)) return T4B_ERR_UNSUPPORTED;
    const bool has_zp = Z != nullptr;
    const int KW = K / 8;
    const int gw = group / 8;
    if (M > 16) return T4B_ERR_UNSUPPORTED;
    if ((K % 128) != 0 || !aligned(A, 16)) return T4B_ERR_UNSUPPORTED;
    for (int j = 0; j < np; ++j) {
        if ((N[j] % 8) != 0 || !aligned(W[j], 16) || !aligned(S[j], 16) || (has_zp && !aligned(Z[j], 16)))
            return T4B_ERR_UNSUPPORTED;
    }
    const int MT = (M <= 8) ? 1 : 2;
    const int warps = (MT == 1) ? Shape<1>::kWarps : Shape<2>::kWarps;
    const int rows_narrow = 16 * warps, rows_wide = 8 * warps, rows_split = 32 * warps;
    // a flush block (8 or 16 word rows) and a scale box (rows_wide rows) must
    // each lie in one group
    auto box_rows = [&](int rows) { return rows % gw == 0 ? rows / gw : (gw % rows == 0 ? 1 : 0); };
    if (!(gw == 8 || gw >= 16) || !box_rows(rows_wide) || !box_rows(rows_narrow)) return T4B_ERR_UNSUPPORTED;
    DecodeParams p;
    p.A = static_cast<const uint16_t*>(A);
    p.M = M; p.K = K; p.KW = KW;
    p.split = (box_rows(rows_split) && M <= 4) ? 1 : 0;         // split groups use 2 batch columns per row
    const int pad_rows = p.split ? rows_split : rows_narrow;       // a split stage may run past KW
    p.KWp = (KW + pad_rows - 1) / pad_rows * pad_rows;
    // Column tiles of each projection and the CTAs (at most one per SM) that
    // share them: with more tiles than SMs, every projection gets a CTA and
    // each further CTA goes to the projection with the most tiles per CTA
    // (a CTA's stages are proportional to its tiles, K being common).
    const int sms = sm_count();
    int T[kMaxProj], G[kMaxProj];
    long long t_total = 0;
    for (int j = 0; j < np; ++j) {
        T[j] = (N[j] + kBoxCols - 1) / kBoxCols;
        t_total += T[j];
    }
    // Every CTA stages all of A (M * K * 2 bytes).  Past M * K = 32768 that
    // only pays when each SM has at least one whole column tile to spend it
    // on; narrower shapes go to the K-split stream kernel.
    if ((long long)M * K > 32768 && t_total < sms) return T4B_ERR_UNSUPPORTED;
    int used = 0;
    if (t_total <= sms) {
        for (int j = 0; j < np; ++j) G[j] = T[j];
        used = (int)t_total;
    } else {
        if (np > sms) return T4B_ERR_UNSUPPORTED;
        for (int j = 0; j < np; ++j) G[j] = 1;
        used = np;
        while (used < sms) {
            int best = -1;
            for (int j = 0; j < np; ++j)
                if (G[j] < T[j] && (best < 0 || (long long)T[j] * G[best] > (long long)T[best] * G[j])) best = j;
            if (best < 0) break;
            ++G[best];
            ++used;
        }
    }
    for (int j = 0; j < np; ++j)
        if ((long long)T[j] * G[j] >= (1ll << 32)) return T4B_ERR_UNSUPPORTED;
    p.nproj = np;
    p.proj_g0[0] = 0;
    for (int j = 0; j < kMaxProj; ++j) {
        const bool in = j < np;
        p.proj_g0[j + 1] = p.proj_g0[j] + (in ? G[j] : 0);
        p.proj_T[j] = in ? T[j] : 0;
        p.proj_N[j] = in ? N[j] : 0;
        p.proj_C[j] = (in && C) ? static_cast<uint16_t*>(C[j]) : nullptr;
        p.proj_coloff[j] = (in && gather) ? (col_offsets ? col_offsets[j] : gather->col_offset) : 0;
    }
    p.T = (int)t_total;
    p.G = used;
    p.N = N[0];
    p.C = p.proj_C[0];
    p.gw = gw;
    p.gw_shift = -1;
    if ((gw & (gw - 1)) == 0) {
        int sh = 0;
        while ((1 << sh) < gw) ++sh;
        p.gw_shift = sh;
    }
    p.fb = (gw == 8) ? 8 : 16;
    p.sbr_wide = box_rows(rows_wide);
    p.sbr_narrow = box_rows(rows_narrow);
    p.sbr_split = p.split ? box_rows(rows_split) : 1;
    p.s_bytes = std::max(std::max(p.sbr_wide * 128, p.sbr_narrow * 64), p.sbr_split * 32);
    p.s_wide = (KW + rows_wide - 1) / rows_wide;
    p.s_narrow = (KW + rows_narrow - 1) / rows_narrow;
    p.s_split = (KW + rows_split - 1) / rows_split;
    p.act_bytes = M * (p.KWp + 2) * 16;
    p.sum_floats = (p.KWp / p.fb) * 8 * MT;
    p.red_floats = 2 * warps * 32 * (M | 1);  // two buffers, row stride M | 1 (see the group epilogue)
    p.kwdiv = make_fastdiv((uint32_t)p.KWp);
    p.world = 1;
    p.rank = 0;
    p.n_total = N[0];
    p.col_offset = 0;
    p.barrier = 0;
    p.gout = nullptr;
    p.counter = nullptr;
    for (int g = 0; g < 8; ++g) p.recv[g] = nullptr;
    if (gather) {
        p.world = gather->world;
        p.rank = gather->rank;
        p.n_total = gather->n_total;
        p.col_offset = gather->col_offset;
        p.barrier = gather->barrier ? 1 : 0;
        p.gout = static_cast<uint32_t*>(gather->out);
        p.counter = gather->counter;
        for (int g = 0; g < p.world; ++g) p.recv[g] = static_cast<unsigned long long*>(gather->recv[g]);
    }
    const int weight_bytes = warps * 2048;
    p.slot_bytes = (weight_bytes + p.s_bytes * (has_zp ? 2 : 1) + 1023) / 1024 * 1024;
    const size_t fixed = 1024 + (size_t)p.act_bytes + 4 * (size_t)(p.sum_floats + p.red_floats) + kMaxStages * 16 + 8 + 16;
    // one CTA per SM with the deepest ring shared memory allows
    const size_t budget = smem_budget();
    int stages = fixed < budget ? (int)((budget - fixed) / p.slot_bytes) : 0;
    if (stages > kMaxStages) stages = kMaxStages;
    if (stages < 2) return T4B_ERR_UNSUPPORTED;
    if (ctas)
        for (int j = 0; j < np; ++j) ctas[j] = G[j];
    if (plan_only) return T4B_OK;
    p.stages = stages;
    // Every stage the ring holds is fetched before the previous kernel ends:
    // with one CTA per SM nothing of the next kernel competes for the copy
    // engine, and the deeper the early fetch the less of the stream is left
    // once the activations are in.
    p.early = stages;
    const size_t smem = fixed + (size_t)stages * p.slot_bytes;

    if (np == 1) {
        DecodeMaps<1> maps;
        if (!make_proj_maps(maps.proj[0], W[0], S[0], has_zp ? Z[0] : nullptr, N[0], K, group, rows_wide, rows_narrow, p))
            return T4B_ERR_UNSUPPORTED;
        return dispatch<1>(is_signed, has_zp, p.fb == 8, MT, maps, p, smem, stream);
    }
    DecodeMaps<kMaxProj> maps;
    for (int j = 0; j < np; ++j)
        if (!make_proj_maps(maps.proj[j], W[j], S[j], has_zp ? Z[j] : nullptr, N[j], K, group, rows_wide, rows_narrow,
                            p))
            return T4B_ERR_UNSUPPORTED;
    for (int j = np; j < kMaxProj; ++j) maps.proj[j] = maps.proj[0];     // never read
    return dispatch<kMaxProj>(is_signed, has_zp, p.fb == 8, MT, maps, p, smem, stream);
}

int gemv_w4_decode(bool is_signed, const void* A, const void* W, const void* S, const void* Z, void* C, int M, int N,
                   int K, int group, cudaStream_t stream) {
    void* Cs[1] = {C};
    return decode_impl(is_signed, A, 1, &W, &S, Z ? &Z : nullptr, Cs, &N, M, K, group, nullptr, stream);
}

int gemv_w4_decode_supported(int M, int N, int K, int group, bool has_zero_points) {
    // a stand-in zero-point pointer: only its presence matters to the plan
    const void* z = reinterpret_cast<const void*>(uintptr_t{256});
    const void* none = nullptr;
    return decode_impl(true, nullptr, 1, &none, &none, has_zero_points ? &z : nullptr, nullptr, &N, M, K, group,
                       nullptr, nullptr, true);
}

int gemv_w4_decode_grouped(bool is_signed, const void* A, int np, const void* const* W, const void* const* S,
                           const void* const* Z, void* const* C, const int* N, int M, int K, int group,
                           cudaStream_t stream) {
    return decode_impl(is_signed, A, np, W, S, Z, C, N, M, K, group, nullptr, stream);
}

int gemv_w4_decode_grouped_plan(int np, const int* N, int M, int K, int group, bool has_zero_points, int* ctas) {
    if (np < 1 || np > kMaxProj) return T4B_ERR_UNSUPPORTED;
    const void* none[kMaxProj] = {};
    const void* z[kMaxProj];
    for (int j = 0; j < kMaxProj; ++j) z[j] = reinterpret_cast<const void*>(uintptr_t{256});
    return decode_impl(true, nullptr, np, none, none, has_zero_points ? z : nullptr, nullptr, N, M, K, group, nullptr,
                       nullptr, true, ctas);
}

// The checks of a T4BGather shared by every projection of a call.
static int check_gather(const T4BGather* g, int M) {
    if (!g || g->world < 2 || g->world > 8 || g->rank < 0 || g->rank >= g->world) return T4B_ERR_INVALID_VALUE;
    if (g->n_total < 2 || (g->n_total & 1)) return T4B_ERR_INVALID_VALUE;     // whole column pairs
    if ((long long)M * g->n_total >= (1ll << 31)) return T4B_ERR_INVALID_VALUE;
    if (!g->out || !g->counter) return T4B_ERR_NULL_POINTER;
    if (reinterpret_cast<uintptr_t>(g->out) & 3) return T4B_ERR_MISALIGNED;
    for (int r = 0; r < g->world; ++r) {
        if (!g->recv[r]) return T4B_ERR_NULL_POINTER;
        if (reinterpret_cast<uintptr_t>(g->recv[r]) & 7) return T4B_ERR_MISALIGNED;
    }
    return T4B_OK;
}

// Columns [off, off + N) of the group buffer: whole column pairs inside it.
static bool gather_columns_ok(const T4BGather* g, int off, int N) {
    return off >= 0 && (long long)off + N <= g->n_total && ((off | N) & 1) == 0;
}

int gemv_w4_decode_gather(bool is_signed, const void* A, const void* W, const void* S, const void* Z, int M, int N,
                          int K, int group, const T4BGather* g, cudaStream_t stream) {
    const int st = check_gather(g, M);
    if (st != T4B_OK) return st;
    if (!gather_columns_ok(g, g->col_offset, N)) return T4B_ERR_INVALID_VALUE;
    return decode_impl(is_signed, A, 1, &W, &S, Z ? &Z : nullptr, nullptr, &N, M, K, group, g, stream);
}

int gemv_w4_decode_gather_grouped(bool is_signed, const void* A, int np, const void* const* W, const void* const* S,
                                  const void* const* Z, const int* N, const int* col_offsets, int M, int K, int group,
                                  const T4BGather* g, cudaStream_t stream) {
    const int st = check_gather(g, M);
    if (st != T4B_OK) return st;
    if (np < 1 || np > kMaxProj) return T4B_ERR_INVALID_VALUE;
    for (int j = 0; j < np; ++j)
        if (!gather_columns_ok(g, col_offsets[j], N[j])) return T4B_ERR_INVALID_VALUE;
    return decode_impl(is_signed, A, np, W, S, Z, nullptr, N, M, K, group, g, stream, false, nullptr, col_offsets);
}

}  // namespace t4b
