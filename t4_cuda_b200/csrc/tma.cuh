// TMA, mbarrier and programmatic-dependent-launch helpers for sm_100a.
//
// No TMA load here is a cluster multicast: every copy reads this GPU's own
// memory into this CTA's shared memory only.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace t4b {

// ------------------------------------------------------------------ host side
// 2-D tiled tensor map over a row-major matrix of 4-byte elements
// (rows x cols, row pitch = cols * 4 bytes) with a box of box_cols x box_rows
// and 128-byte swizzle.  Out-of-range elements of a box read as zero.
// Returns false if the driver entry point is unavailable or encoding fails.
bool make_tmap_u32_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows,
                      uint32_t box_cols);

// Same for 2-byte elements (fp16), box_cols * 2 must be <= 128 bytes.
bool make_tmap_f16_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows,
                      uint32_t box_cols);

// General form: element type u32 or fp16, swizzle 0 / 32 / 64 / 128 bytes
// (a box row may not be wider than the swizzle span), L2 promotion
// 0 / 64 / 128 / 256 bytes.
bool make_tmap_2d_ex(CUtensorMap* map, bool fp16, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows,
                     uint32_t box_cols, int swizzle_bytes, int l2_promotion_bytes);

// 3-D view of a row-major matrix of 4-byte elements (rows x cols) as
// (tile_cols, floor(cols / tile_cols), rows) -- whole tiles only -- with a box
// of tile_cols x box_tiles x box_rows and 128-byte swizzle.  tile_cols * 4
// must be exactly 128: the swizzle lays every box row out at a 128-byte
// pitch, so a narrower inner dimension would take more shared memory than
// the box's bytes.  One box row is box_tiles * tile_cols consecutive elements
// of a matrix row, so a box of adjacent tiles is fetched as wide contiguous
// rows; it lands in shared memory as [box_rows][box_tiles * 128 B] with the
// 16-byte units of each 128-byte line permuted by the line's index (mod 8).
// Returns false if encoding fails.
bool make_tmap_tiles_3d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t tile_cols,
                        uint32_t box_tiles, uint32_t box_rows);

// --------------------------------------------------------------- device side
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

// Make mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait on an mbarrier phase: gives up after `limit_ns` nanoseconds
// and returns false (the caller records an error and unwinds) instead of
// spinning forever.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (global_timer_ns() - t0 > limit_ns) return false;
    }
}

// 2-D TMA load of one box into shared memory, completion signalled on `bar`
// as transaction bytes.  Coordinates: x = column (innermost), y = row.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// 3-D TMA load of one box (coordinates innermost first).
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
            smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue now / wait until the previous kernel's results are visible.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait_prior_grid() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Named barrier over `nthreads` threads (a multiple of 32), id 1..15.
__device__ __forceinline__ void named_barrier(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

}  // namespace t4b
