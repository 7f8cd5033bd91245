// Torch binding of the fused matmul ops -- the role of src/bindings.cpp:64-250
// in the reference (a torch C++ extension), in front of this library's C ABI.
//
// The decode path calls a fused op once per projection per token, so the
// per-call host cost bounds a step run from Python: this binding does the
// argument checks, the output allocation and the launch in C++ (the same
// checks, in the same order and with the same messages, as the Python path in
// ops.py, which mirrors bindings.cpp).  It calls the C ABI through function
// pointers taken from the library that ops.py has loaded (init), so the
// process has one copy of the library's state (kernel choices, caches).
#include <torch/extension.h>

#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

// t4b_fused_w4a16_gemm_{u4,s4}(A, W, S, Z, C, M, N, K, group, stream)
using FusedFn = int (*)(const void*, const void*, const void*, const void*, void*, int, int, int, int, void*);
// t4b_fused_w4a16_gemv_allgather(A, W, S, Z, M, N, K, group, is_signed, gather, stream)
using AllgatherFn = int (*)(const void*, const void*, const void*, const void*, int, int, int, int, int, const void*,
                            void*);
// t4b_fused_w4a16_gemv_allgather_grouped(A, n, W[], S[], Z[], N[], col_offsets[], M, K, group, is_signed,
//                                        gather, stream)
using AllgatherGroupedFn = int (*)(const void*, int, const void* const*, const void* const*, const void* const*,
                                   const int*, const int*, int, int, int, int, const void*, void*);
// t4b_fused_w4a16_gemm_grouped(A, n, W[], S[], Z[], C[], N[], M, K, group, is_signed, stream)
using GroupedFn = int (*)(const void*, int, const void* const*, const void* const*, const void* const*, void* const*,
                          const int*, int, int, int, int, void*);
using StatusStringFn = const char* (*)(int);
using LastCudaErrorFn = int (*)();

FusedFn g_u4 = nullptr, g_s4 = nullptr;
AllgatherFn g_allgather = nullptr;
GroupedFn g_grouped = nullptr;
AllgatherGroupedFn g_allgather_grouped = nullptr;
StatusStringFn g_status_string = nullptr;
LastCudaErrorFn g_last_cuda_error = nullptr;
PyObject* g_error_class = nullptr;      // t4_cuda_b200._lib.T4BError (a RuntimeError)

[[noreturn]] void fail(const std::string& msg) { throw std::runtime_error(msg); }

// A non-zero status as the library's error class, with the message of _lib.check.
[[noreturn]] void raise_status(int st, const char* op) {
    std::string msg = std::string(op) + ": " + (g_status_string ? g_status_string(st) : "error") + " (status " +
                      std::to_string(st);
    const int cuda = (st == 5 && g_last_cuda_error) ? g_last_cuda_error() : 0;
    if (cuda) msg += ", cudaError " + std::to_string(cuda);
    msg += ")";
    PyErr_SetString(g_error_class ? g_error_class : PyExc_RuntimeError, msg.c_str());
    throw pybind11::error_already_set();
}

// (N,) / (1, N) / (G, N) -> number of rows G, with the checks of ops._group_rows.
int64_t group_rows(const torch::Tensor& t, int64_t N, int64_t K, const char* what, int64_t word_values) {
    const int64_t d = t.dim();
    if (d == 1) {
        if (t.numel() != N)
            fail(std::string(what) + " of shape (N,) must have N=" + std::to_string(N) + " elements, got " +
                 std::to_string(t.numel()));
        return 1;
    }
    if (d != 2) fail(std::string(what) + " must be 1-D (N,) or 2-D (K/group, N)");
    if (t.size(1) != N)
        fail(std::string(what) + " must have N=" + std::to_string(N) + " columns, got " + std::to_string(t.size(1)));
    const int64_t G = t.size(0);
    if (G < 1 || K % G)
        fail(std::string(what) + ": " + std::to_string(G) + " groups must divide K=" + std::to_string(K));
    if ((K / G) % word_values)
        fail(std::string(what) + ": group size K/" + std::to_string(G) + "=" + std::to_string(K / G) +
             " must be a multiple of " + std::to_string(word_values));
    return G;
}

// Contiguous tensor whose data pointer is 16-byte aligned (copy if not).
torch::Tensor aligned16(const torch::Tensor& t) {
    torch::Tensor c = t.is_contiguous() ? t : t.contiguous();
    if (reinterpret_cast<uintptr_t>(c.data_ptr()) % 16) c = c.clone();
    return c;
}

bool has_values(const c10::optional<torch::Tensor>& z) { return z.has_value() && z->defined() && z->numel() > 0; }

struct WShape {
    int64_t M, N, K, G;
    bool has_zp;
};

// ops._check_w: the checks of bindings.cpp:64-132 after A's device check.
WShape check_w(const torch::Tensor& A, const torch::Tensor& W, const torch::Tensor& S,
               const c10::optional<torch::Tensor>& Zopt) {
    if (!W.is_cuda()) fail("W_packed must be a CUDA tensor");
    if (!S.is_cuda()) fail("scales must be a CUDA tensor");
    const bool has_zp = has_values(Zopt);
    if (has_zp) {
        if (!Zopt->is_cuda()) fail("zero_points must be a CUDA tensor");
        if (Zopt->scalar_type() != torch::kFloat16) fail("zero_points must be FP16");
    }
    if (A.scalar_type() != torch::kFloat16) fail("A must be FP16");
    if (W.scalar_type() != torch::kInt32) fail("W_packed must be Int32");
    if (S.scalar_type() != torch::kFloat16) fail("scales must be FP16");
    if (A.dim() != 2) fail("A must be a 2-D (M, K) tensor");
    if (W.dim() != 2) fail("W_packed must be a 2-D (K/8, N) tensor");
    const auto dev = A.device();
    if (W.device() != dev || S.device() != dev || (has_zp && Zopt->device() != dev))
        fail("all tensors must be on the same device");
    const int64_t M = A.size(0), K = A.size(1), N = W.size(1);
    if (M <= 0 || N <= 0 || K <= 0) fail("Dimensions M, N, K must be positive");
    if (K % 8) fail("K must be a multiple of 8 (8 INT4 values per int32 word)");
    if (W.size(0) != K / 8)
        fail("W_packed must have K/8=" + std::to_string(K / 8) + " rows, got " + std::to_string(W.size(0)));
    const int64_t G = group_rows(S, N, K, "scales", 8);
    if (has_zp && group_rows(*Zopt, N, K, "zero_points", 8) != G) fail("zero_points must have the same shape as scales");
    return {M, N, K, G, has_zp};
}

torch::Tensor contig(const torch::Tensor& t) { return t.is_contiguous() ? t : t.contiguous(); }

// ops._fused: C = A @ dequant_w4(W_packed), bindings.cpp:64-132.
torch::Tensor fused_w4(FusedFn fn, const char* name, const torch::Tensor& A, const torch::Tensor& W,
                       const torch::Tensor& S, const c10::optional<torch::Tensor>& Zopt) {
    if (!fn) fail("t4_cuda_b200 torch binding not initialised");
    if (!A.is_cuda()) fail("A must be a CUDA tensor");
    const WShape w = check_w(A, W, S, Zopt);
    const torch::Tensor A_ = aligned16(A);
    const torch::Tensor W_ = contig(W);
    const torch::Tensor S_ = contig(S);
    torch::Tensor Z_;
    if (w.has_zp) Z_ = contig(*Zopt);
    const auto dev = A.device();
    const c10::cuda::CUDAGuard guard(dev);
    torch::Tensor C = torch::empty({w.M, w.N}, A.options());
    const int st = fn(A_.data_ptr(), W_.data_ptr(), S_.data_ptr(), w.has_zp ? Z_.data_ptr() : nullptr, C.data_ptr(),
                      (int)w.M, (int)w.N, (int)w.K, (int)(w.K / w.G),
                      c10::cuda::getCurrentCUDAStream(dev.index()).stream());
    if (st) raise_status(st, name);
    return C;
}

constexpr int kGroupedMax = 4;      // T4B_GROUPED_MAX

// ops._fused_grouped: the projections of W_list that read A, in one call.
std::vector<torch::Tensor> fused_w4a16_gemm_grouped(const torch::Tensor& A, const std::vector<torch::Tensor>& Ws,
                                                    const std::vector<torch::Tensor>& Ss,
                                                    const c10::optional<std::vector<c10::optional<torch::Tensor>>>& Zs,
                                                    bool is_signed) {
    if (!g_grouped) fail("t4_cuda_b200 torch binding not initialised");
    const int n = (int)Ws.size();
    if (n < 1 || n > kGroupedMax)
        fail("a grouped call takes 1 to " + std::to_string(kGroupedMax) + " projections, got " + std::to_string(n));
    if ((int)Ss.size() != n || (Zs.has_value() && (int)Zs->size() != n))
        fail("W_packed, scales and zero_points lists must have the same length");
    if (!A.is_cuda()) fail("A must be a CUDA tensor");
    WShape w[kGroupedMax];
    for (int j = 0; j < n; ++j) {
        const c10::optional<torch::Tensor> z = Zs.has_value() ? (*Zs)[j] : c10::nullopt;
        w[j] = check_w(A, Ws[j], Ss[j], z);
    }
    for (int j = 1; j < n; ++j)
        if (w[j].G != w[0].G) fail("every projection of a grouped call must have the same group size");
    for (int j = 1; j < n; ++j)
        if (w[j].has_zp != w[0].has_zp)
            fail("zero_points must be given for every projection of a grouped call or for none");
    const bool has_zp = w[0].has_zp;
    const torch::Tensor A_ = aligned16(A);
    torch::Tensor W_[kGroupedMax], S_[kGroupedMax], Z_[kGroupedMax];
    const void *wp[kGroupedMax], *sp[kGroupedMax], *zp[kGroupedMax];
    void* cp[kGroupedMax];
    int Ns[kGroupedMax];
    const auto dev = A.device();
    const c10::cuda::CUDAGuard guard(dev);
    std::vector<torch::Tensor> C;
    C.reserve(n);
    for (int j = 0; j < n; ++j) {
        W_[j] = contig(Ws[j]);
        S_[j] = contig(Ss[j]);
        wp[j] = W_[j].data_ptr();
        sp[j] = S_[j].data_ptr();
        if (has_zp) {
            Z_[j] = contig(*(*Zs)[j]);
            zp[j] = Z_[j].data_ptr();
        }
        C.push_back(torch::empty({w[j].M, w[j].N}, A.options()));
        cp[j] = C.back().data_ptr();
        Ns[j] = (int)w[j].N;
    }
    const int st = g_grouped(A_.data_ptr(), n, wp, sp, has_zp ? zp : nullptr, cp, Ns, (int)w[0].M, (int)w[0].K,
                             (int)(w[0].K / w[0].G), is_signed ? 1 : 0,
                             c10::cuda::getCurrentCUDAStream(dev.index()).stream());
    if (st) raise_status(st, "t4b_fused_w4a16_gemm_grouped");
    return C;
}

torch::Tensor fused_w4a16_gemm_u4(const torch::Tensor& A, const torch::Tensor& W, const torch::Tensor& S,
                                  const c10::optional<torch::Tensor>& Z) {
    return fused_w4(g_u4, "t4b_fused_w4a16_gemm_u4", A, W, S, Z);
}

torch::Tensor fused_w4a16_gemm_s4(const torch::Tensor& A, const torch::Tensor& W, const torch::Tensor& S,
                                  const c10::optional<torch::Tensor>& Z) {
    return fused_w4(g_s4, "t4b_fused_w4a16_gemm_s4", A, W, S, Z);
}

// One call of a fused-gather group (shard.P2PGatherGroup.__call__): the
// launches of its projections in order, from a table the group builds once --
// int64 [n, 8]: W, scales, zero points (0: none), N (this rank's columns), K,
// group size, is_signed, address of the projection's T4BGather.  x: the
// group's activations, contiguous fp16 [M, K] on the current device.
void allgather_group(const torch::Tensor& x, const torch::Tensor& table, int64_t M) {
    if (!g_allgather) fail("t4_cuda_b200 torch binding not initialised");
    if (!x.is_cuda() || x.scalar_type() != torch::kFloat16 || !x.is_contiguous() || x.dim() != 2 || x.size(0) != M)
        fail("the fused gather group takes contiguous fp16 activations of " + std::to_string(M) + " rows");
    if (table.is_cuda() || table.scalar_type() != torch::kInt64 || table.dim() != 2 || table.size(1) != 8 ||
        !table.is_contiguous())
        fail("gather table must be a contiguous CPU int64 [n, 8] tensor");
    const int64_t* t = table.data_ptr<int64_t>();
    const c10::cuda::CUDAGuard guard(x.device());
    void* stream = c10::cuda::getCurrentCUDAStream(x.device().index()).stream();
    const void* a = x.data_ptr();
    for (int64_t i = 0; i < table.size(0); ++i, t += 8) {
        const int st = g_allgather(a, reinterpret_cast<const void*>(t[0]), reinterpret_cast<const void*>(t[1]),
                                   reinterpret_cast<const void*>(t[2]), (int)M, (int)t[3], (int)t[4], (int)t[5],
                                   (int)t[6], reinterpret_cast<const void*>(t[7]), stream);
        if (st) raise_status(st, "t4b_fused_w4a16_gemv_allgather");
    }
}

// One call of a fused-gather group made as one grouped launch
// (shard.P2PGatherGroup with grouped=True): int64 table [n, 9] -- W, scales,
// zero points (0: none), N, K, group size, is_signed, address of the group's
// T4BGather, the projection's first column in the group buffer.
void allgather_grouped(const torch::Tensor& x, const torch::Tensor& table, int64_t M) {
    if (!g_allgather_grouped) fail("t4_cuda_b200 torch binding not initialised");
    if (!x.is_cuda() || x.scalar_type() != torch::kFloat16 || !x.is_contiguous() || x.dim() != 2 || x.size(0) != M)
        fail("the fused gather group takes contiguous fp16 activations of " + std::to_string(M) + " rows");
    const int64_t n = table.size(0);
    if (table.is_cuda() || table.scalar_type() != torch::kInt64 || table.dim() != 2 || table.size(1) != 9 ||
        !table.is_contiguous() || n < 1 || n > kGroupedMax)
        fail("grouped gather table must be a contiguous CPU int64 [n, 9] tensor, 1 <= n <= 4");
    const int64_t* t = table.data_ptr<int64_t>();
    const void *wp[kGroupedMax], *sp[kGroupedMax], *zp[kGroupedMax];
    int Ns[kGroupedMax], offs[kGroupedMax];
    for (int64_t i = 0; i < n; ++i) {
        const int64_t* r = t + 9 * i;
        wp[i] = reinterpret_cast<const void*>(r[0]);
        sp[i] = reinterpret_cast<const void*>(r[1]);
        zp[i] = reinterpret_cast<const void*>(r[2]);
        Ns[i] = (int)r[3];
        offs[i] = (int)r[8];
    }
    const c10::cuda::CUDAGuard guard(x.device());
    void* stream = c10::cuda::getCurrentCUDAStream(x.device().index()).stream();
    const int st = g_allgather_grouped(x.data_ptr(), (int)n, wp, sp, t[2] ? zp : nullptr, Ns, offs, (int)M, (int)t[4],
                                       (int)t[5], (int)t[6], reinterpret_cast<const void*>(t[7]), stream);
    if (st) raise_status(st, "t4b_fused_w4a16_gemv_allgather_grouped");
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.doc() = "torch binding of t4_cuda_b200's fused W4A16 ops and fused-gather group calls (the hot paths)";
    m.def(
        "init",
        [](uintptr_t u4, uintptr_t s4, uintptr_t allgather, uintptr_t grouped, uintptr_t allgather_grouped,
           uintptr_t status_string, uintptr_t last_cuda_error, pybind11::object error_class) {
            g_u4 = reinterpret_cast<FusedFn>(u4);
            g_s4 = reinterpret_cast<FusedFn>(s4);
            g_allgather = reinterpret_cast<AllgatherFn>(allgather);
            g_grouped = reinterpret_cast<GroupedFn>(grouped);
            g_allgather_grouped = reinterpret_cast<AllgatherGroupedFn>(allgather_grouped);
            g_status_string = reinterpret_cast<StatusStringFn>(status_string);
            g_last_cuda_error = reinterpret_cast<LastCudaErrorFn>(last_cuda_error);
            Py_XDECREF(g_error_class);
            g_error_class = error_class.ptr();
            Py_XINCREF(g_error_class);
        },
        "Entry points of the loaded C library (addresses) and the error class.");
    m.def("fused_w4a16_gemm_u4", &fused_w4a16_gemm_u4, "C = A @ dequant_u4(W_packed)", pybind11::arg("A"),
          pybind11::arg("W_packed"), pybind11::arg("scales"), pybind11::arg("zero_points"));
    m.def("fused_w4a16_gemm_s4", &fused_w4a16_gemm_s4, "C = A @ dequant_s4(W_packed)", pybind11::arg("A"),
          pybind11::arg("W_packed"), pybind11::arg("scales"), pybind11::arg("zero_points"));
    m.def("fused_w4a16_gemm_grouped", &fused_w4a16_gemm_grouped,
          "[A @ dequant(W) for W in W_list]: projections that read the same activation, in one call",
          pybind11::arg("A"), pybind11::arg("W_list"), pybind11::arg("scales_list"),
          pybind11::arg("zero_points_list"), pybind11::arg("is_signed"));
    m.def("allgather_grouped", &allgather_grouped, "One fused-gather group call as one grouped launch, from its table",
          pybind11::arg("x"), pybind11::arg("table"), pybind11::arg("M"));
    m.def("allgather_group", &allgather_group, "The launches of one fused-gather group call, from its table",
          pybind11::arg("x"), pybind11::arg("table"), pybind11::arg("M"));
}
