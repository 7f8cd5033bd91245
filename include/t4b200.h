/*
 * t4b200.h -- C ABI of the B200 (sm_100a) W4A16 / INT3 quantized-matmul library.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (passed as void*, a cudaStream_t; NULL = the legacy default stream),
 * enqueues its kernels asynchronously and returns a status code (T4B_OK = 0).
 * Nothing throws across this boundary.  The caller owns every input and output
 * buffer; the W4A16 matmul additionally uses a scratch workspace that the
 * library allocates itself (cudaMalloc, never freed), once per (device,
 * stream), on the first call that needs it -- also inside CUDA-graph capture,
 * where it allocates at capture time -- and grows when a call needs more.
 * Element types: "f16" = IEEE binary16 (uint16 storage), "words" = uint32
 * (int32 in torch) holding packed weights.
 *
 * Each function replaces one launcher of the reference project
 * (kridaydave/t4-cuda); the citation names the reference declaration it stands
 * in for and the pybind op that called it (src/bindings.cpp:252-260).
 */
#ifndef T4B200_H
#define T4B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
enum {
    T4B_OK = 0,
    T4B_ERR_INVALID_VALUE = 1,   /* a size, group or mode argument is out of range      */
    T4B_ERR_NULL_POINTER = 2,    /* a required pointer is NULL                          */
    T4B_ERR_MISALIGNED = 3,      /* a pointer breaks the alignment the op documents     */
    T4B_ERR_UNSUPPORTED = 4,     /* shape/option combination this build does not serve */
    T4B_ERR_CUDA = 5,            /* a CUDA runtime call or kernel launch failed         */
    T4B_ERR_SCRATCH_LIMIT = 6    /* problem needs more than the fixed scratch array of
                                    t4b_fused_w4a16_gemv_noalloc                        */
};

/* Dequantization arithmetic (argument `mode` of the t4b_dequantize_* calls). */
enum {
    T4B_MODE_CONTRACT = 0,  /* fp16_rn(fp32_rn((q - z) * s)): what the reference tests assert */
    T4B_MODE_MAGIC = 1      /* bit-exact with the reference GPU kernels' LOP3 + fma.rn.f16x2    */
};

/* Human-readable text for a status code (static storage). */
const char* t4b_status_string(int status);

/* The cudaError_t of the most recent T4B_ERR_CUDA on the calling thread (0 if none). */
int t4b_last_cuda_error(void);

/* Library ABI version: (major << 16) | minor. */
int t4b_version(void);

/* Reads (and, if `clear`, resets) the library's device error words on the
 * current device -- the decode GEMV's, the prefill GEMMs' (INT4 / FP8 and INT3)
 * and the INT3 GEMV's (one each per device), the allocation-free GEMV's (in its fixed scratch
 * array) and the one
 * in the workspace kept for `stream` (if any), ORed: bit 0 = a kernel gave up
 * a bounded wait (its output is then invalid).  Synchronizes `stream`; do not
 * call while the stream is being captured.  No counterpart in the reference,
 * which has no device-side error reporting. */
int t4b_device_error(void* stream, unsigned* out, int clear);

/* Bytes of the workspace this library holds for `stream` on the current
 * device (0 if it has made none): the split-tile GEMV and the split-K GEMM
 * cudaMalloc one on their first call on a stream.  A diagnostic with no
 * counterpart in the reference, for callers that must know whether the library
 * allocated device memory. */
int t4b_workspace_bytes(void* stream, size_t* bytes);

/* Kernel selection for the W4A16 matmul (argument of t4b_set_gemv_kernel). */
enum {
    T4B_GEMV_AUTO = 0,     /* best kernel that applies: for M <= 16 the resident-activation
                              decode kernel, then the TMA-streamed split-tile kernel; for
                              M > 16 the tcgen05 GEMM (CTA pairs when M > 128); else generic */
    T4B_GEMV_GENERIC = 1,  /* always the generic register-streaming kernel (for comparison)  */
    T4B_GEMV_STREAM = 2,   /* the TMA-streamed split-tile kernel where it applies, else generic */
    T4B_GEMV_TC_SINGLE = 3 /* as AUTO, but M > 16 always on the single-CTA tcgen05 kernel     */
};
/* Sets the process-wide choice; returns the previous one (-1: bad argument).
 * No counterpart in the reference (it has a single kernel). */
int t4b_set_gemv_kernel(int which);

/* Kernel choice for the INT3 GEMV: 0 = the register-streaming kernel (the
 * default); 1 = the warp-specialized TMA-ring kernel where it applies
 * (N % 4 == 0, W 16-byte and scales 8-byte aligned), else register streaming;
 * 2 = register streaming at every M; 3 = the tcgen05 INT3 GEMM at every M
 * where it takes the shape (else as 0).  Under 0 and 1, M > 16 runs on the
 * tcgen05 INT3 GEMM where it takes the shape (an even group_size >= 64,
 * N % 8 == 0, 16-byte aligned operands).  Returns the previous choice (-1:
 * bad argument).  No counterpart in the reference. */
int t4b_set_int3_kernel(int which);

/* ---- flat dequantization ----------------------------------------------
 * out[8*i + j] = dequant(nibble j of words[i], scales[i], zero_points[i]).
 * Scale / zero point are per WORD (lop3_dequant.cu:19-21); num_scales and
 * num_zero_points are either num_words or 1 (broadcast); num_zero_points = 0
 * (zero_points may then be NULL) means zero.  out holds num_words*8 f16
 * (u4, s4), num_words*10 (s3) or num_words*4 (fp8).  num_words may be 0.
 */

/* replaces launch_lop3_dequant_u4 (src/kernels/lop3_dequant.h:126-127), op dequantize_u4 */
int t4b_dequantize_u4(const void* words, const void* scales, const void* zero_points,
                      void* out, int64_t num_words, int64_t num_scales,
                      int64_t num_zero_points, int mode, void* stream);

/* replaces launch_lop3_dequant_s4 (src/kernels/lop3_dequant.h:129-130), op dequantize_s4 */
int t4b_dequantize_s4(const void* words, const void* scales, const void* zero_points,
                      void* out, int64_t num_words, int64_t num_scales,
                      int64_t num_zero_points, int mode, void* stream);

/* replaces launch_lop3_dequant_s3 (src/kernels/lop3_dequant.h:132-133), op dequantize_s3 */
int t4b_dequantize_s3(const void* words, const void* scales, const void* zero_points,
                      void* out, int64_t num_words, int64_t num_scales,
                      int64_t num_zero_points, int mode, void* stream);

/* replaces launch_lop3_dequant_fp8 (src/kernels/lop3_dequant.h:135-136), op dequantize_fp8 */
int t4b_dequantize_fp8(const void* words, const void* scales, void* out,
                       int64_t num_words, int64_t num_scales, int mode, void* stream);

/* ---- fused W4A16 matmul -----------------------------------------------
 * C[M, N] (f16, row-major) = A[M, K] (f16, row-major) x dequant(W)[K, N]
 * with W_packed int32 [K/8, N] row-major, K row 8*kw + j in nibble j of word
 * (kw, n).  scales / zero_points are f16 [K/group_size, N] row-major; the
 * reference's per-column (1, N) tensors are group_size = K.  zero_points may
 * be NULL (zero).  Requirements: M, N >= 1; K >= 8, K % 8 == 0;
 * group_size % 8 == 0 and K % group_size == 0.  Weights are rounded to f16
 * by the contract rule; products and sums are fp32.
 */

/* replaces launch_fused_w4a16_gemm_u4 (src/kernels/fused_w4a16_gemm.h:24-31), op fused_w4a16_gemm_u4 */
int t4b_fused_w4a16_gemm_u4(const void* A, const void* W_packed, const void* scales,
                            const void* zero_points, void* C, int M, int N, int K,
                            int group_size, void* stream);

/* replaces launch_fused_w4a16_gemm_s4 (src/kernels/fused_w4a16_gemm.h:39-46), op fused_w4a16_gemm_s4 */
int t4b_fused_w4a16_gemm_s4(const void* A, const void* W_packed, const void* scales,
                            const void* zero_points, void* C, int M, int N, int K,
                            int group_size, void* stream);

/* Projections that read the same activation, in one call: C[j] (f16
 * [M, N[j]]) = A x dequant(W_packed[j]) for j < n (1 <= n <= T4B_GROUPED_MAX),
 * all with the same K, group_size and signedness (is_signed: s4, else u4).
 * zero_points is NULL (no zero points) or n pointers, all set.  No
 * counterpart in the reference, whose op takes one projection (a layer's
 * q/k/v or gate/up are n calls of fused_w4a16_gemm_{u4,s4}); the results
 * match those n calls within the ops' tolerance.  Where the decode kernel
 * takes the shapes (M <= 16 under T4B_GEMV_AUTO / TC_SINGLE) the projections
 * run as one launch whose CTAs are shared out by column tiles; otherwise the
 * call makes the n single calls itself. */
#define T4B_GROUPED_MAX 4
int t4b_fused_w4a16_gemm_grouped(const void* A, int n, const void* const* W_packed,
                                 const void* const* scales, const void* const* zero_points,
                                 void* const* C, const int* N, int M, int K, int group_size,
                                 int is_signed, void* stream);

/* T4B_OK and the CTAs of each projection (ctas[j], j < n) of the one launch
 * t4b_fused_w4a16_gemm_grouped makes for these shapes, or T4B_ERR_UNSUPPORTED
 * when it would make single calls instead; launches nothing, but reads the
 * current device's SM count. */
int t4b_fused_w4a16_gemm_grouped_plan(int n, const int* N, int M, int K, int group_size,
                                      int has_zero_points, int* ctas);

/* FP8-E4M3 weight GEMM.  No counterpart in the reference, which has only the
 * flat dequantizer of this format (launch_lop3_dequant_fp8,
 * src/kernels/lop3_dequant.h:135-136): the fused path for it.
 * C[M, N] (f16) = A[M, K] (f16) x (E4M3(W) * s)[K, N]; W_packed int32 [K/4, N],
 * byte j of word (kw, n) = K row 4 kw + j; scales f16 [K/group_size, N].  The
 * weight is f16(e4m3 * s) with exact E4M3 decoding (subnormals are values,
 * 0x7F / 0xFF are NaN); products and sums fp32.  Runs the tcgen05 GEMM for any
 * M >= 1; needs K % 64 == 0, group_size % 64 == 0, N % 8 == 0 and 16-byte
 * aligned pointers (else T4B_ERR_UNSUPPORTED / T4B_ERR_MISALIGNED). */
int t4b_fused_w8a16_gemm_fp8(const void* A, const void* W_packed, const void* scales, void* C,
                             int M, int N, int K, int group_size, void* stream);

/* Allocation-free decode GEMV.  No counterpart in the reference: an addition
 * for callers that cannot allocate device memory while they run -- a serving
 * engine that reserves all of HBM for its own pool at start-up, or a host
 * runtime that forbids cudaMalloc once it is serving.  Same math and result as
 * t4b_fused_w4a16_gemm_s4 (is_signed != 0) or _u4 (is_signed == 0) for
 * M <= 16, but its scratch (split-tile partial sums, flags, an error word)
 * lives in a fixed 4 MiB array inside this library, present on every GPU that
 * loads it until the process exits; it never calls cudaMalloc or cudaFree.
 * Extra requirements: M <= 16, N % 4 == 0, W_packed 16-byte and scales /
 * zero_points 8-byte aligned, and (group_size / 8) a multiple of 8 or >= K / 8
 * (else T4B_ERR_UNSUPPORTED); a shape whose partial sums do not fit in 4 MiB
 * returns T4B_ERR_SCRATCH_LIMIT (Llama-3-8B projection shapes fit up to M = 16).
 * The first call on each device looks up the array's device address (with that
 * device current); make that first call before any stream capture.  Every call
 * shares the one array: calls that overlap on the GPU (different streams,
 * concurrent graph replays) race and give wrong results.  Each call clears the
 * array's flags on `stream` before its kernel; its error word (bit 0: a bounded
 * wait gave up and C is invalid) stays set until t4b_device_error clears it. */
int t4b_fused_w4a16_gemv_noalloc(const void* A, const void* W_packed, const void* scales,
                                 const void* zero_points, void* C, int M, int N, int K,
                                 int group_size, int is_signed, void* stream);

/* ---- column-sharded decode GEMV with a fused all-gather over peer memory ---
 * No counterpart in the reference (it has no multi-GPU code).  Rank `rank` of
 * `world` GPUs (one process each) holds columns of a projection; instead of a
 * GEMV followed by an all-gather collective, the decode kernel stores each
 * pair of its output columns, with the call's epoch, as one 64-bit word into
 * every rank's receive buffer (device pointers of peer memory, opened with
 * t4b_ipc_open).  The words validate themselves, so no fence or flag is
 * needed.  Several calls (projections that share an activation) form a group;
 * its last call (barrier = 1) ends only when the whole group has arrived in
 * this rank's receive buffer, and then `out` holds the [M, n_total] output.
 *   recv[g]      rank g's receive buffer: 2 halves (epoch parity) of
 *                M x n_total/2 64-bit words, zero at start
 *   out          this rank's gathered output, [M, n_total] fp16 (local)
 *   counter      this rank's two uint32 (zero at start): CTAs done, epoch
 *   col_offset   first column this rank writes (even); n_total even
 * Every rank makes the same sequence of calls on the same buffers; a call's
 * epoch is the group's count of completed groups + 1.  Waits are bounded
 * (2 s); a rank that gives up sets the device error word.  Returns
 * T4B_ERR_UNSUPPORTED (nothing launched) for shapes the decode kernel does not
 * take; the caller then falls back to its collective. */
typedef struct {
    void* recv[8];
    void* out;
    unsigned* counter;
    int world, rank, n_total, col_offset, barrier;
} T4BGather;

/* T4B_OK when t4b_fused_w4a16_gemv_allgather takes a shape (this rank's N
 * columns), T4B_ERR_UNSUPPORTED when it does not; launches nothing, but reads
 * the current device's SM count. */
int t4b_fused_w4a16_gemv_allgather_supported(int M, int N, int K, int group_size, int has_zero_points);

int t4b_fused_w4a16_gemv_allgather(const void* A, const void* W_packed, const void* scales,
                                   const void* zero_points, int M, int N, int K, int group_size,
                                   int is_signed, const T4BGather* gather, void* stream);

/* The n projections of a group (1 <= n <= T4B_GROUPED_MAX, same K, group_size,
 * signedness and presence of zero points) as one launch of the decode kernel
 * with the fused all-gather: projection j stores its N[j] columns at columns
 * [col_offsets[j], col_offsets[j] + N[j]) of the group buffer (even offsets
 * and widths); gather->col_offset is not used, gather->barrier as above (1
 * when this call is the group's last).  No counterpart in the reference.
 * Returns T4B_ERR_UNSUPPORTED (nothing launched) where the decode kernel does
 * not take the shapes as one launch (t4b_fused_w4a16_gemm_grouped_plan says
 * which); the caller then makes one t4b_fused_w4a16_gemv_allgather call per
 * projection. */
int t4b_fused_w4a16_gemv_allgather_grouped(const void* A, int n, const void* const* W_packed,
                                           const void* const* scales, const void* const* zero_points,
                                           const int* N, const int* col_offsets, int M, int K,
                                           int group_size, int is_signed, const T4BGather* gather,
                                           void* stream);

/* Device memory another process on this node can map: cudaMalloc'd and zeroed
 * (t4b_ipc_alloc), its 64-byte handle (t4b_ipc_handle), the peer's mapping of
 * a handle (t4b_ipc_open) and their release. */
int t4b_ipc_alloc(size_t bytes, void** ptr);
int t4b_ipc_free(void* ptr);
int t4b_ipc_handle(void* ptr, void* handle64);
int t4b_ipc_open(const void* handle64, void** ptr);
int t4b_ipc_close(void* ptr);

/* ---- H17 fused INT3 GEMV ------------------------------------------------
 * C[M, N] (f16) = A[M, K] (f16) x dequant_s3(W)[K, N], W_packed int32 [K/10, N],
 * element i of word (kw, n) = K row 10*kw + i at bits 3i..3i+2.
 * scales / zero_points f16 [ceil(K/group_size), N]; zero_points may be NULL.
 * Requirements: M, N >= 1; K >= 10, K % 10 == 0; group_size >= 10 (so that a
 * word spans at most two groups; smaller groups return T4B_ERR_UNSUPPORTED).
 */

/* replaces launch_h17_gemv_s3 (src/kernels/h17_mega_kernel.h:22-30), op fused_h17_gemv_s3 */
int t4b_fused_h17_gemv_s3(const void* A, const void* W_packed, const void* scales,
                          const void* zero_points, void* C, int M, int N, int K,
                          int group_size, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* T4B200_H */
