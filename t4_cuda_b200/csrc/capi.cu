// Library-wide C ABI plumbing: status strings, the per-thread CUDA error
// record, the cached per-device SM count used to size grids, the per-stream
// workspace of the streaming GEMV, and TMA tensor-map encoding.
#include <cstring>

#include "common.cuh"
#include "tma.cuh"
#include "workspace.h"

#include <cudaTypedefs.h>

#include <map>
#include <mutex>
#include <utility>

namespace t4b {

namespace {
thread_local int g_last_cuda_error = 0;
std::mutex g_sm_mutex;
int g_sm_counts[64] = {0};

struct WsBuf {
    void* base = nullptr;
    size_t counter_words = 0;
    size_t part_floats = 0;
};
std::mutex g_ws_mutex;
std::map<std::pair<int, cudaStream_t>, WsBuf> g_ws;

constexpr size_t kHeaderBytes = 256;
size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
}  // namespace

int record_cuda_error(cudaError_t err) {
    g_last_cuda_error = (int)err;
    return T4B_ERR_CUDA;
}

int sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    {
        std::lock_guard<std::mutex> lock(g_sm_mutex);
        if (g_sm_counts[dev]) return g_sm_counts[dev];
    }
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    std::lock_guard<std::mutex> lock(g_sm_mutex);
    g_sm_counts[dev] = n;
    return n;
}

int ensure_dynamic_smem(const void* kernel, int bytes, SmemLimit* limit) {
    static std::mutex mu;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return record_cuda_error(e);
    if (dev < 0 || dev >= 64) return T4B_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(mu);
    if (limit->bytes[dev] >= bytes) return T4B_OK;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return record_cuda_error(e);
    limit->bytes[dev] = bytes;
    return T4B_OK;
}

int acquire_workspace(cudaStream_t stream, size_t counter_words, size_t part_floats, Workspace* ws) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return record_cuda_error(e);
    std::lock_guard<std::mutex> lock(g_ws_mutex);
    WsBuf& buf = g_ws[{dev, stream}];
    if (!buf.base || buf.counter_words < counter_words || buf.part_floats < part_floats) {
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        e = cudaStreamIsCapturing(stream, &cap);
        if (e != cudaSuccess) return record_cuda_error(e);
        const bool capturing = cap != cudaStreamCaptureStatusNone;
        // Grow with headroom; the previous buffer may still be in use by queued
        // kernels (or by a captured graph), so it is kept, never freed --
        // growth is rare and bounded.
        const size_t cw = round_up(std::max(counter_words * 2, std::max(buf.counter_words, (size_t)65536)), 64);
        const size_t pf = round_up(std::max(part_floats * 2, std::max(buf.part_floats, (size_t)(1 << 20))), 64);
        const size_t bytes = kHeaderBytes + cw * 4 + pf * 4;
        void* p = nullptr;
        if (capturing) {
            // First use on a stream that is being captured into a CUDA graph
            // (torch captures on a side stream of its own).  A cudaMalloc is
            // allowed during capture once this thread's capture mode is
            // relaxed; the buffer is zeroed on a private stream and waited for
            // here, outside the graph, and it is never freed, so the graph's
            // kernels can rely on it at every replay.
            cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
            e = cudaThreadExchangeStreamCaptureMode(&mode);
            if (e != cudaSuccess) return record_cuda_error(e);
            cudaStream_t zs = nullptr;
            e = cudaMalloc(&p, bytes);
            if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&zs, cudaStreamNonBlocking);
            if (e == cudaSuccess) e = cudaMemsetAsync(p, 0, kHeaderBytes + cw * 4, zs);
            if (e == cudaSuccess) e = cudaStreamSynchronize(zs);
            if (zs) cudaStreamDestroy(zs);
            cudaThreadExchangeStreamCaptureMode(&mode);      // back to the caller's mode
            if (e != cudaSuccess) return record_cuda_error(e);
        } else {
            e = cudaMalloc(&p, bytes);
            if (e != cudaSuccess) return record_cuda_error(e);
            e = cudaMemsetAsync(p, 0, kHeaderBytes + cw * 4, stream);
            if (e != cudaSuccess) return record_cuda_error(e);
        }
        buf.base = p;
        buf.counter_words = cw;
        buf.part_floats = pf;
    }
    char* base = static_cast<char*>(buf.base);
    ws->error = reinterpret_cast<unsigned*>(base);
    ws->counters = reinterpret_cast<unsigned*>(base + kHeaderBytes);
    ws->part = reinterpret_cast<float*>(base + kHeaderBytes + buf.counter_words * 4);
    return T4B_OK;
}

// ------------------------------------------------------------- tensor maps
namespace {
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

bool make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t esize, const void* base, uint64_t rows,
                  uint64_t cols, uint32_t box_rows, uint32_t box_cols) {
    auto fn = encode_fn();
    if (!fn) return false;
    if ((cols * esize) % 16 != 0 || (reinterpret_cast<uintptr_t>(base) % 16) != 0) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * esize};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace

bool make_tmap_u32_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows,
                      uint32_t box_cols) {
    return make_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, base, rows, cols, box_rows, box_cols);
}

bool make_tmap_f16_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows,
                      uint32_t box_cols) {
    return make_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, rows, cols, box_rows, box_cols);
}

namespace {

// Encoded tensor maps, per host thread, keyed by every encoding parameter.  A
// decode call encodes six to eight maps, and a model calls the same weights
// every token: the driver's encode is then the largest host cost of a call.
// A map depends on nothing but its key (base address, shape, box, swizzle,
// L2 promotion), so a hit is exactly what a fresh encode would produce.
struct TmapKey {
    const void* base;
    uint64_t rows, cols;
    uint32_t box_rows, box_cols;
    int swizzle, l2, fp16;
    bool operator==(const TmapKey& o) const {
        return base == o.base && rows == o.rows && cols == o.cols && box_rows == o.box_rows &&
               box_cols == o.box_cols && swizzle == o.swizzle && l2 == o.l2 && fp16 == o.fp16;
    }
};

struct TmapEntry {
    TmapKey key;
    CUtensorMap map;
    bool valid;
};

constexpr int kTmapCacheSize = 512;      // direct-mapped
thread_local TmapEntry t_tmap_cache[kTmapCacheSize];

uint32_t tmap_hash(const TmapKey& k) {
    uint64_t h = reinterpret_cast<uintptr_t>(k.base) * 0x9E3779B97F4A7C15ull;
    h ^= (k.rows * 0xC2B2AE3D27D4EB4Full) + (k.cols << 17) + ((uint64_t)k.box_rows << 40) + ((uint64_t)k.box_cols << 29);
    h ^= (uint64_t)(k.swizzle * 7 + k.l2 * 131 + k.fp16 * 65537);
    h ^= h >> 29;
    return (uint32_t)(h % kTmapCacheSize);
}

}  // namespace

int max_active_clusters(const void* kernel, int smem, int threads, int ks, ClusterCapacityCache* cache) {
    if (ks < 2 || ks > 8) return 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64) {
        const int c = cache->n[dev][ks].load(std::memory_order_relaxed);
        if (c > 0) return c - 1;
    }
    int n = 0;
    if (ensure_dynamic_smem(kernel, smem, &cache->limit) == T4B_OK) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(1, 1, (unsigned)ks);
        cfg.blockDim = dim3((unsigned)threads, 1, 1);
        cfg.dynamicSmemBytes = (size_t)smem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = (unsigned)ks;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess) {
            cudaGetLastError();
            n = 0;
        }
    }
    if (dev >= 0 && dev < 64) cache->n[dev][ks].store(n + 1, std::memory_order_relaxed);
    return n;
}

bool make_tmap_2d_ex(CUtensorMap* map, bool fp16, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows,
                     uint32_t box_cols, int swizzle_bytes, int l2_promotion_bytes) {
    const TmapKey key{base, rows, cols, box_rows, box_cols, swizzle_bytes, l2_promotion_bytes, fp16 ? 1 : 0};
    TmapEntry& slot = t_tmap_cache[tmap_hash(key)];
    if (slot.valid && slot.key == key) {
        *map = slot.map;
        return true;
    }
    slot.valid = false;
    auto fn = encode_fn();
    if (!fn) return false;
    const uint32_t esize = fp16 ? 2 : 4;
    if ((cols * esize) % 16 != 0 || (reinterpret_cast<uintptr_t>(base) % 16) != 0) return false;
    if ((box_cols * esize) % 16 != 0) return false;
    CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_NONE;
    if (swizzle_bytes == 32) sw = CU_TENSOR_MAP_SWIZZLE_32B;
    else if (swizzle_bytes == 64) sw = CU_TENSOR_MAP_SWIZZLE_64B;
    else if (swizzle_bytes == 128) sw = CU_TENSOR_MAP_SWIZZLE_128B;
    else if (swizzle_bytes != 0) return false;
    if (swizzle_bytes && box_cols * esize > (uint32_t)swizzle_bytes) return false;
    CUtensorMapL2promotion l2 = CU_TENSOR_MAP_L2_PROMOTION_NONE;
    if (l2_promotion_bytes == 64) l2 = CU_TENSOR_MAP_L2_PROMOTION_L2_64B;
    else if (l2_promotion_bytes == 128) l2 = CU_TENSOR_MAP_L2_PROMOTION_L2_128B;
    else if (l2_promotion_bytes == 256) l2 = CU_TENSOR_MAP_L2_PROMOTION_L2_256B;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * esize};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    if (fn(map, fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(base), dims,
           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, l2, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    slot.key = key;
    slot.map = *map;
    slot.valid = true;
    return true;
}

bool make_tmap_tiles_3d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t tile_cols,
                        uint32_t box_tiles, uint32_t box_rows) {
    // cached with the 2-D maps; fp16 = 2 marks this kind of map
    const TmapKey key{base, rows, cols, box_rows, box_tiles * 1024u + tile_cols, 128, 256, 2};
    TmapEntry& slot = t_tmap_cache[tmap_hash(key)];
    if (slot.valid && slot.key == key) {
        *map = slot.map;
        return true;
    }
    slot.valid = false;
    auto fn = encode_fn();
    if (!fn) return false;
    // the view holds the whole tiles of a row (a trailing partial tile is left out)
    if (tile_cols == 0 || cols < tile_cols || tile_cols * 4 != 128) return false;
    if ((cols * 4) % 16 != 0 || (reinterpret_cast<uintptr_t>(base) % 16) != 0) return false;
    cuuint64_t dims[3] = {tile_cols, cols / tile_cols, rows};   // floor: whole tiles only
    cuuint64_t strides[2] = {(cuuint64_t)tile_cols * 4, cols * 4};
    cuuint32_t box[3] = {tile_cols, box_tiles, box_rows};
    cuuint32_t estr[3] = {1, 1, 1};
    if (fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<void*>(base), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    slot.key = key;
    slot.map = *map;
    slot.valid = true;
    return true;
}

}  // namespace t4b

extern "C" {

const char* t4b_status_string(int status) {
    switch (status) {
        case T4B_OK: return "ok";
        case T4B_ERR_INVALID_VALUE: return "invalid value (size, group size or mode out of range)";
        case T4B_ERR_NULL_POINTER: return "a required pointer is NULL";
        case T4B_ERR_MISALIGNED: return "a pointer is not aligned as the operation requires";
        case T4B_ERR_UNSUPPORTED: return "shape or option not supported by this build";
        case T4B_ERR_CUDA: return "CUDA runtime error (see t4b_last_cuda_error)";
        case T4B_ERR_SCRATCH_LIMIT: return "problem too large for the fixed 4 MiB scratch of the allocation-free GEMV";
        default: return "unknown status";
    }
}

int t4b_last_cuda_error(void) { return t4b::g_last_cuda_error; }

int t4b_ipc_alloc(size_t bytes, void** ptr) {
    if (!ptr || bytes == 0) return T4B_ERR_INVALID_VALUE;
    *ptr = nullptr;
    cudaError_t e = cudaMalloc(ptr, bytes);
    if (e == cudaSuccess) e = cudaMemset(*ptr, 0, bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();   // zeroed before any peer can map it
    return e == cudaSuccess ? T4B_OK : t4b::record_cuda_error(e);
}

int t4b_ipc_free(void* ptr) {
    cudaError_t e = cudaFree(ptr);
    return e == cudaSuccess ? T4B_OK : t4b::record_cuda_error(e);
}

int t4b_ipc_handle(void* ptr, void* handle64) {
    if (!ptr || !handle64) return T4B_ERR_NULL_POINTER;
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "64-byte IPC handle");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
    if (e != cudaSuccess) return t4b::record_cuda_error(e);
    memcpy(handle64, &h, sizeof(h));
    return T4B_OK;
}

int t4b_ipc_open(const void* handle64, void** ptr) {
    if (!handle64 || !ptr) return T4B_ERR_NULL_POINTER;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle64, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? T4B_OK : t4b::record_cuda_error(e);
}

int t4b_ipc_close(void* ptr) {
    cudaError_t e = cudaIpcCloseMemHandle(ptr);
    return e == cudaSuccess ? T4B_OK : t4b::record_cuda_error(e);
}

int t4b_version(void) { return (1 << 16) | 1; }

int t4b_device_error(void* stream, unsigned* out, int clear) {
    if (!out) return T4B_ERR_NULL_POINTER;
    *out = 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // the decode GEMV keeps one word per device
    unsigned decode = 0;
    int st = t4b::decode_device_error(s, &decode, clear != 0);
    if (st != T4B_OK) return st;
    *out = decode;
    // so does the prefill GEMM
    unsigned gemm = 0;
    st = t4b::gemm_tc_device_error(s, &gemm, clear != 0);
    if (st != T4B_OK) return st;
    *out |= gemm;
    // the INT3 GEMV's ring form
    unsigned int3w = 0;
    st = t4b::int3_device_error(s, &int3w, clear != 0);
    if (st != T4B_OK) return st;
    *out |= int3w;
    // the INT3 prefill GEMM
    unsigned int3g = 0;
    st = t4b::int3_tc_device_error(s, &int3g, clear != 0);
    if (st != T4B_OK) return st;
    *out |= int3g;
    // and the allocation-free GEMV, in its fixed scratch array
    unsigned fixed = 0;
    st = t4b::static_scratch_error(s, &fixed, clear != 0);
    if (st != T4B_OK) return st;
    *out |= fixed;
    // the split-tile GEMV keeps one in the workspace of each stream
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return t4b::record_cuda_error(e);
    void* base = nullptr;
    {
        std::lock_guard<std::mutex> lock(t4b::g_ws_mutex);
        auto it = t4b::g_ws.find({dev, s});
        if (it == t4b::g_ws.end()) return T4B_OK;
        base = it->second.base;
    }
    unsigned word = 0;
    e = cudaMemcpyAsync(&word, base, sizeof(unsigned), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess && clear) e = cudaMemsetAsync(base, 0, sizeof(unsigned), s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return t4b::record_cuda_error(e);
    *out |= word;
    return T4B_OK;
}

int t4b_workspace_bytes(void* stream, size_t* bytes) {
    if (!bytes) return T4B_ERR_NULL_POINTER;
    *bytes = 0;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return t4b::record_cuda_error(e);
    std::lock_guard<std::mutex> lock(t4b::g_ws_mutex);
    auto it = t4b::g_ws.find({dev, static_cast<cudaStream_t>(stream)});
    if (it != t4b::g_ws.end() && it->second.base)
        *bytes = t4b::kHeaderBytes + (it->second.counter_words + it->second.part_floats) * 4;
    return T4B_OK;
}

}  // extern "C"
