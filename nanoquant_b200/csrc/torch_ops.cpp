// Thin PyTorch dispatcher layer over the nq_b200 C ABI.
//
// Registers the reference's op namespace `binary_kernels` with the reference schemas
// (src/nanoquant/kernel/pybind.cpp:83-125), so NanoQuantLinear._prepare_kernel and
// get_kernel_function (src/nanoquant/kernel/utils.py:33-48) bind these kernels
// unchanged, plus the `nq_b200` namespace for packing and the explicit GEMV / GEMM.
// Every op has a CUDA and a Meta implementation.  Kernels run on the current CUDA
// stream of the input's device; nothing synchronises (except pack_signs with
// check=True, which must read the invalid-value count back).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <map>
#include <tuple>
#include <mutex>
#include <optional>
#include <string>
#include <utility>
#include <vector>

#include "../../include/nq_b200.h"
#include "../../include/nq_decoder.h"

namespace {

#define NQ_TORCH_CHECK(call)                                                                          \
    do {                                                                                              \
        const int nq_st_ = (call);                                                                    \
        TORCH_CHECK(nq_st_ == NQ_OK, "nq_b200: ", nq_status_string(nq_st_), ": ", nq_last_error_message()); \
    } while (0)

#define CHECK_CUDA_CONT(x, st)                                                        \
    do {                                                                              \
        TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor");                      \
        TORCH_CHECK((x).is_contiguous(), #x " must be contiguous");                   \
        TORCH_CHECK((x).scalar_type() == (st), #x " must be ", c10::toString(st), " tensor"); \
    } while (0)

int dtype_code(at::ScalarType st) {
    if (st == at::kHalf) return NQ_DTYPE_F16;
    if (st == at::kBFloat16) return NQ_DTYPE_BF16;
    TORCH_CHECK(false, "Support only Half or BFloat16");
}

int order_code(const std::string &m) {
    if (m == "lsb_first") return NQ_BITS_LSB_FIRST;
    if (m == "half2") return NQ_BITS_HALF2;
    TORCH_CHECK_VALUE(false, "Unsupported method: '", m, "'. Supported methods are 'lsb_first', 'half2'.");
}

cudaStream_t cur_stream(const at::Tensor &t) { return c10::cuda::getCurrentCUDAStream(t.device().index()).stream(); }

// Zero-initialised workspace per (device, stream, slot), grown on demand and kept for the
// life of the process (its control block must start zeroed; kernels keep it so).  Slot 0
// serves the linears, slot 1 decode attention.
at::Tensor workspace_for(const at::Tensor &like, size_t bytes, int slot = 0) {
    static std::mutex mu;
    static std::map<std::tuple<int, cudaStream_t, int>, at::Tensor> cache;
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_tuple((int)like.device().index(), cur_stream(like), slot);
    auto it = cache.find(key);
    if (it == cache.end() || (size_t)it->second.numel() < bytes) {
        size_t cap = bytes < (1u << 20) ? (1u << 20) : bytes;
        at::Tensor ws = at::zeros({(int64_t)cap}, like.options().dtype(at::kByte));
        cache[key] = ws;
        return ws;
    }
    return it->second;
}

// reference parameter_sweep sets (src/nanoquant/kernel/cuda/gemv_kernel.cu:351-354)
void check_choice(const char *name, int64_t v, std::initializer_list<int64_t> allowed) {
    bool found = false;
    std::string choices;
    for (int64_t a : allowed) {
        if (a == v) found = true;
        if (!choices.empty()) choices += ", ";
        choices += std::to_string(a);
    }
    TORCH_CHECK_VALUE(found, name, " should be one of [", choices, "], but ", v, " was given");
}

int64_t gemm_min_rows() {
    static int64_t v = [] {
        const char *e = std::getenv("NQ_GEMM_MIN_ROWS");
        return e ? std::atoll(e) : (int64_t)33;
    }();
    return v;
}

struct LayerArgs {
    at::Tensor x, s2, vbits, s1;
    std::optional<at::Tensor> smid;
    at::Tensor ubits;
    int64_t rows, in_f, rank, out_f;
};

LayerArgs check_layer(const at::Tensor &x, const at::Tensor &s2, const at::Tensor &vbits,
                      const std::optional<at::Tensor> &smid, const at::Tensor &ubits, const at::Tensor &s1) {
    const auto st = x.scalar_type();
    dtype_code(st);
    CHECK_CUDA_CONT(x, st);
    CHECK_CUDA_CONT(s2, st);
    CHECK_CUDA_CONT(s1, st);
    CHECK_CUDA_CONT(vbits, at::kInt);
    CHECK_CUDA_CONT(ubits, at::kInt);
    TORCH_CHECK(x.dim() == 1 || x.dim() == 2, "x must be 1-D or 2-D [rows, in_features]");
    LayerArgs a{x, s2, vbits, s1, std::nullopt, ubits, 0, 0, 0, 0};
    a.rows = x.dim() == 1 ? 1 : x.size(0);
    a.in_f = x.size(-1);
    a.rank = vbits.size(0);
    a.out_f = s1.numel();
    TORCH_CHECK(vbits.dim() == 2 && vbits.size(1) == (a.in_f + 31) / 32, "V planes must be [rank, ceil(in/32)]");
    TORCH_CHECK(ubits.dim() == 2 && ubits.size(0) == a.out_f && ubits.size(1) == (a.rank + 31) / 32,
                "U planes must be [out, ceil(rank/32)]");
    TORCH_CHECK(s2.numel() == a.in_f, "scale_pre size mismatch");
    if (smid.has_value() && smid->defined()) {
        CHECK_CUDA_CONT((*smid), st);
        TORCH_CHECK(smid->numel() == a.rank, "scale_l size mismatch");
        a.smid = *smid;
    }
    for (const at::Tensor *t : {&s2, &vbits, &ubits, &s1})
        TORCH_CHECK(t->device() == x.device(), "all tensors must be on the same device");
    return a;
}

at::Tensor run_gemv(const LayerArgs &a) {
    c10::cuda::CUDAGuard guard(a.x.device());
    auto y = at::empty({a.rows, a.out_f}, a.x.options());
    const size_t wsb = nq_gemv_workspace_bytes(a.rows, a.rank);
    at::Tensor ws = workspace_for(a.x, wsb);
    NQ_TORCH_CHECK(nq_gemv(dtype_code(a.x.scalar_type()), a.x.data_ptr(), a.rows, a.in_f, a.s2.data_ptr(),
                           a.vbits.data_ptr<int32_t>(), a.rank, a.smid ? a.smid->data_ptr() : nullptr,
                           a.ubits.data_ptr<int32_t>(), a.out_f, a.s1.data_ptr(), y.data_ptr(), ws.data_ptr(),
                           (size_t)ws.numel(), cur_stream(a.x)));
    return y;
}

at::Tensor run_gemm(const LayerArgs &a, bool precise) {
    c10::cuda::CUDAGuard guard(a.x.device());
    auto y = at::empty({a.rows, a.out_f}, a.x.options());
    const size_t wsb = nq_gemm_workspace_bytes(a.rows, a.rank);
    at::Tensor ws = at::empty({(int64_t)wsb}, a.x.options().dtype(at::kByte));
    NQ_TORCH_CHECK(nq_gemm(dtype_code(a.x.scalar_type()), a.x.data_ptr(), a.rows, a.in_f, a.s2.data_ptr(),
                           a.vbits.data_ptr<int32_t>(), a.rank, a.smid ? a.smid->data_ptr() : nullptr,
                           a.ubits.data_ptr<int32_t>(), a.out_f, a.s1.data_ptr(), precise ? 1 : 0, y.data_ptr(),
                           ws.data_ptr(), wsb, cur_stream(a.x)));
    return y;
}

bool gemm_ok(const LayerArgs &a) {
    return a.rows >= gemm_min_rows() && a.in_f % 8 == 0 &&
           (reinterpret_cast<uintptr_t>(a.x.data_ptr()) & 15) == 0;
}

// GEMM precision: bf16 layers keep T as a bf16 hi/lo pair (rounding T to bf16 alone costs about
// 2e-3 rel-L2); fp16 layers round T once to fp16, the reference's own intermediate (gemm.cpp:119),
// well inside 1e-3, with one stage-2 MMA per K step instead of two.
at::Tensor forward_auto(const LayerArgs &a) {
    at::Tensor y = gemm_ok(a) ? run_gemm(a, a.x.scalar_type() == at::kBFloat16) : run_gemv(a);
    return a.x.dim() == 1 ? y.squeeze(0) : y;
}

// ------------------------------------------------------------------ Marlin layout (reference gemm kernel type)
// Inverses of the reference's scale permutations (src/nanoquant/kernel/utils.py:207-210).
at::Tensor marlin_unperm_in(const at::Tensor &s) { return s.reshape({-1, 4, 2, 2}).permute({0, 2, 1, 3}).reshape({-1}); }
at::Tensor marlin_unperm_out(const at::Tensor &s) { return s.reshape({-1, 4, 4, 2}).permute({0, 2, 1, 3}).reshape({-1}); }

at::Tensor marlin_to_half2_t(const at::Tensor &words, int64_t n_out, int64_t k_red) {
    CHECK_CUDA_CONT(words, at::kInt);
    TORCH_CHECK(words.dim() == 2 && words.size(0) * 16 == k_red && words.size(1) * 2 == n_out,
                "Marlin words must be [k_red/16, n_out/2]");
    c10::cuda::CUDAGuard guard(words.device());
    auto planes = at::empty({n_out, (k_red + 31) / 32}, words.options());
    NQ_TORCH_CHECK(nq_marlin_to_half2(words.data_ptr<int32_t>(), n_out, k_red, planes.data_ptr<int32_t>(),
                                      cur_stream(words)));
    return planes;
}

// The reference's marlin_onebit_check_and_alloc (gemm.cpp:37-56): same checks, same messages.
void marlin_check(const at::Tensor &A, const at::Tensor &B, const std::optional<at::Tensor> &s_in,
                  const std::optional<at::Tensor> &s_out, const at::Tensor &workspace) {
    constexpr int64_t kMinMaxPar = 32;  // MARLIN_MIN_MAX_PAR
    TORCH_CHECK(A.scalar_type() == at::kHalf || A.scalar_type() == at::kBFloat16,
                "Unsupported dtype: Marlin only supports Half and BFloat16");
    TORCH_CHECK(A.dim() == 2 && B.dim() == 2, "x and the weight must be 2-D");
    const int64_t prob_n = B.size(1) * 2, prob_k = A.size(1);
    TORCH_CHECK(prob_k == B.size(0) * 16, "k dimension mismatch");
    TORCH_CHECK(!s_in.has_value() || s_in->size(0) == prob_k, "s_in size mismatch");
    TORCH_CHECK(!s_out.has_value() || s_out->size(0) == prob_n, "s_out size mismatch");
    TORCH_CHECK(workspace.numel() >= prob_n / 128 * kMinMaxPar, "workspace too small");
}

at::Tensor marlin_onebit_forward_cuda(const at::Tensor &x, const at::Tensor &weight,
                                      const std::optional<at::Tensor> &scale_g,
                                      const std::optional<at::Tensor> &scale_h, at::Tensor &workspace) {
    marlin_check(x, weight, scale_g, scale_h, workspace);
    CHECK_CUDA_CONT(x, x.scalar_type());
    c10::cuda::CUDAGuard guard(x.device());
    const int64_t m = x.size(0), k = x.size(1), n = weight.size(1) * 2;
    at::Tensor planes = marlin_to_half2_t(weight, n, k);
    at::Tensor s_in = scale_g.has_value() ? marlin_unperm_in(scale_g->to(x.scalar_type())).contiguous()
                                          : at::ones({k}, x.options());
    at::Tensor s_out;
    if (scale_h.has_value()) s_out = marlin_unperm_out(scale_h->to(x.scalar_type())).contiguous();
    auto y = at::empty({m, n}, x.options());
    if (m == 0) return y;
    at::Tensor ws = at::zeros({(int64_t)nq_gemm_onebit_workspace_bytes()}, x.options().dtype(at::kByte));
    NQ_TORCH_CHECK(nq_gemm_onebit(dtype_code(x.scalar_type()), x.data_ptr(), m, k, s_in.data_ptr(),
                                  planes.data_ptr<int32_t>(), n, s_out.defined() ? s_out.data_ptr() : nullptr,
                                  y.data_ptr(), ws.data_ptr(), (size_t)ws.numel(), cur_stream(x)));
    return y;
}

at::Tensor marlin_onebit_forward_meta(const at::Tensor &x, const at::Tensor &weight,
                                      const std::optional<at::Tensor> &scale_g,
                                      const std::optional<at::Tensor> &scale_h, at::Tensor &workspace) {
    marlin_check(x, weight, scale_g, scale_h, workspace);
    return at::empty({x.size(0), weight.size(1) * 2}, x.options());
}

// marlin_nanoquant_cuda (gemm.cpp:112-122) is two marlin_onebit calls: imm = x V (s_in = scale_g,
// s_out = scale_l), y = imm U (s_out = scale_h).  Here the two factors are converted to HALF2
// planes and the layer runs as one NanoQuant layer of rank = the padded rank: the GEMV for up to
// 32 rows, the tcgen05 GEMM above (fp16: T rounded once to fp16 like the reference's imm).
at::Tensor marlin_nanoquant_forward_cuda(const at::Tensor &x, const at::Tensor &weight_u, const at::Tensor &weight_v,
                                         const std::optional<at::Tensor> &scale_g,
                                         const std::optional<at::Tensor> &scale_l,
                                         const std::optional<at::Tensor> &scale_h, at::Tensor &workspace) {
    marlin_check(x, weight_u, scale_g, scale_l, workspace);
    const int64_t rank = weight_u.size(1) * 2;
    TORCH_CHECK(rank == weight_v.size(0) * 16, "k dimension mismatch");
    TORCH_CHECK(!scale_h.has_value() || scale_h->size(0) == weight_v.size(1) * 2, "s_out size mismatch");
    TORCH_CHECK(workspace.numel() >= weight_v.size(1) * 2 / 128 * 32, "workspace too small");
    CHECK_CUDA_CONT(x, x.scalar_type());
    c10::cuda::CUDAGuard guard(x.device());
    const int64_t in_f = x.size(1), out_f = weight_v.size(1) * 2;
    at::Tensor vb = marlin_to_half2_t(weight_u, rank, in_f);
    at::Tensor ub = marlin_to_half2_t(weight_v, out_f, rank);
    const auto dt = x.scalar_type();
    at::Tensor s2 = scale_g.has_value() ? marlin_unperm_in(scale_g->to(dt)).contiguous() : at::ones({in_f}, x.options());
    at::Tensor s1 = scale_h.has_value() ? marlin_unperm_out(scale_h->to(dt)).contiguous() : at::ones({out_f}, x.options());
    std::optional<at::Tensor> smid;
    if (scale_l.has_value()) smid = marlin_unperm_out(scale_l->to(dt)).contiguous();
    if (x.size(0) == 0) return at::empty({0, out_f}, x.options());
    return forward_auto(check_layer(x, s2, vb, smid, ub, s1));
}

at::Tensor marlin_nanoquant_forward_meta(const at::Tensor &x, const at::Tensor &weight_u, const at::Tensor &weight_v,
                                         const std::optional<at::Tensor> &scale_g,
                                         const std::optional<at::Tensor> &scale_l,
                                         const std::optional<at::Tensor> &scale_h, at::Tensor &workspace) {
    marlin_check(x, weight_u, scale_g, scale_l, workspace);
    return at::empty({x.size(0), weight_v.size(1) * 2}, x.options());
}

// ------------------------------------------------------------------ binary_kernels (reference schemas)

at::Tensor nanoquant_dyn_forward_cuda(const at::Tensor &x, const at::Tensor &scale_g, const at::Tensor &Ubits,
                                      const std::optional<at::Tensor> &scale_l, const at::Tensor &Vbits,
                                      const at::Tensor &scale_h, int64_t num_thread_stage1,
                                      int64_t num_thread_stage2, int64_t num_row_per_warp_stage1,
                                      int64_t num_row_per_warp_stage2, int64_t num_acc_stage1,
                                      int64_t num_acc_stage2, int64_t num_pipeline_stage1,
                                      int64_t num_pipeline_stage2) {
    // The tuning knobs select among the reference's template instances; this build
    // chooses its own launch shape but accepts and validates the same values.
    check_choice("n_th1", num_thread_stage1, {64, 128, 256});
    check_choice("n_rpw1", num_row_per_warp_stage1, {1, 2, 4, 8});
    check_choice("n_acc1", num_acc_stage1, {1, 2});
    check_choice("n_pipe1", num_pipeline_stage1, {1, 2, 4, 8, 16});
    check_choice("n_th2", num_thread_stage2, {64, 128, 256});
    check_choice("n_rpw2", num_row_per_warp_stage2, {1, 2, 4, 8});
    check_choice("n_acc2", num_acc_stage2, {1, 2});
    check_choice("n_pipe2", num_pipeline_stage2, {1, 2, 4, 8, 16});
    // Argument names follow the reference op: Ubits = the module's V planes [rank, in/32],
    // scale_l = scale_mid, Vbits = the module's U planes [out, rank/32], scale_h = scale_post.
    return forward_auto(check_layer(x, scale_g, Ubits, scale_l, Vbits, scale_h));
}

at::Tensor nanoquant_dyn_forward_meta(const at::Tensor &x, const at::Tensor &scale_g, const at::Tensor &Ubits,
                                      const std::optional<at::Tensor> &scale_l, const at::Tensor &Vbits,
                                      const at::Tensor &scale_h, int64_t, int64_t, int64_t, int64_t, int64_t,
                                      int64_t, int64_t, int64_t) {
    auto shape = x.sizes().vec();
    shape.back() = scale_h.size(0);
    return at::empty(shape, x.options());
}

// ------------------------------------------------------------------ nq_b200 namespace

at::Tensor pack_signs_cuda(const at::Tensor &signs, const std::string &method, bool check) {
    TORCH_CHECK_TYPE(signs.scalar_type() == at::kChar, "Input tensor must be int8.");
    TORCH_CHECK(signs.is_cuda(), "signs must be a CUDA tensor");
    TORCH_CHECK(signs.dim() == 2, "signs must be 2-D [rows, cols]");
    const int order = order_code(method);
    c10::cuda::CUDAGuard guard(signs.device());
    at::Tensor s = signs.contiguous();
    const int64_t rows = s.size(0), cols = s.size(1);
    auto out = at::empty({rows, (cols + 31) / 32}, s.options().dtype(at::kInt));
    if (rows == 0 || cols == 0) return out;
    at::Tensor bad;
    if (check) bad = at::zeros({1}, s.options().dtype(at::kInt));
    NQ_TORCH_CHECK(nq_pack_signs(s.data_ptr<int8_t>(), rows, cols, order, out.data_ptr<int32_t>(),
                                 check ? bad.data_ptr<int32_t>() : nullptr, cur_stream(s)));
    if (check) {
        const int n = bad.item<int>();
        TORCH_CHECK_VALUE(n == 0, "Cannot pack: factors must contain only -1 and +1 (", n, " other values)");
    }
    return out;
}

at::Tensor pack_marlin_cuda(const at::Tensor &signs, bool check) {
    TORCH_CHECK_TYPE(signs.scalar_type() == at::kChar, "Input tensor must be int8.");
    TORCH_CHECK(signs.is_cuda(), "signs must be a CUDA tensor");
    TORCH_CHECK(signs.dim() == 2, "signs must be 2-D [n_out, k_red]");
    c10::cuda::CUDAGuard guard(signs.device());
    at::Tensor s = signs.contiguous();
    const int64_t n = s.size(0), k = s.size(1);
    TORCH_CHECK_VALUE(n % 64 == 0 && k % 16 == 0, "the Marlin layout needs n_out % 64 == 0 and k_red % 16 == 0, got ",
                      s.sizes());
    auto out = at::empty({k / 16, n / 2}, s.options().dtype(at::kInt));
    if (n == 0 || k == 0) return out;
    at::Tensor bad;
    if (check) bad = at::zeros({1}, s.options().dtype(at::kInt));
    NQ_TORCH_CHECK(nq_pack_marlin(s.data_ptr<int8_t>(), n, k, out.data_ptr<int32_t>(),
                                  check ? bad.data_ptr<int32_t>() : nullptr, cur_stream(s)));
    if (check) {
        const int nb = bad.item<int>();
        TORCH_CHECK_VALUE(nb == 0, "Cannot pack: factors must contain only -1 and +1 (", nb, " other values)");
    }
    return out;
}

at::Tensor pack_marlin_meta(const at::Tensor &signs, bool) {
    return at::empty({signs.size(1) / 16, signs.size(0) / 2}, signs.options().dtype(at::kInt));
}

at::Tensor unpack_marlin_cuda(const at::Tensor &words, int64_t n_out, int64_t k_red) {
    CHECK_CUDA_CONT(words, at::kInt);
    TORCH_CHECK_VALUE(words.dim() == 2 && words.size(0) * 16 == k_red && words.size(1) * 2 == n_out,
                      "Marlin words must be [k_red/16, n_out/2]");
    c10::cuda::CUDAGuard guard(words.device());
    auto out = at::empty({n_out, k_red}, words.options().dtype(at::kChar));
    if (n_out == 0 || k_red == 0) return out;
    NQ_TORCH_CHECK(nq_unpack_marlin(words.data_ptr<int32_t>(), n_out, k_red, out.data_ptr<int8_t>(), cur_stream(words)));
    return out;
}

at::Tensor unpack_marlin_meta(const at::Tensor &words, int64_t n_out, int64_t k_red) {
    return at::empty({n_out, k_red}, words.options().dtype(at::kChar));
}

at::Tensor marlin_to_half2_cuda(const at::Tensor &words, int64_t n_out, int64_t k_red) {
    return marlin_to_half2_t(words, n_out, k_red);
}

at::Tensor marlin_to_half2_meta(const at::Tensor &words, int64_t n_out, int64_t k_red) {
    return at::empty({n_out, (k_red + 31) / 32}, words.options());
}

at::Tensor pack_signs_meta(const at::Tensor &signs, const std::string &method, bool check) {
    order_code(method);
    return at::empty({signs.size(0), (signs.size(1) + 31) / 32}, signs.options().dtype(at::kInt));
}

at::Tensor unpack_signs_cuda(const at::Tensor &packed, int64_t rows, int64_t cols, const std::string &method) {
    TORCH_CHECK_VALUE(packed.dim() == 2, "Unsupported packed tensor format. Expected 2D tensor, got ", packed.dim(),
                      " dimensions.");
    TORCH_CHECK_VALUE(packed.size(0) == rows && packed.size(1) == (cols + 31) / 32,
                      "Unsupported packed tensor shape. Expected (", rows, ", ", (cols + 31) / 32, "), got ",
                      packed.sizes());
    const int order = order_code(method);
    CHECK_CUDA_CONT(packed, at::kInt);
    c10::cuda::CUDAGuard guard(packed.device());
    auto out = at::empty({rows, cols}, packed.options().dtype(at::kChar));
    if (rows == 0 || cols == 0) return out;
    NQ_TORCH_CHECK(nq_unpack_signs(packed.data_ptr<int32_t>(), rows, cols, order, out.data_ptr<int8_t>(),
                                   cur_stream(packed)));
    return out;
}

at::Tensor unpack_signs_meta(const at::Tensor &packed, int64_t rows, int64_t cols, const std::string &method) {
    return at::empty({rows, cols}, packed.options().dtype(at::kChar));
}

at::Tensor repack_signs_cuda(const at::Tensor &packed, int64_t cols, const std::string &src_method,
                             const std::string &dst_method) {
    CHECK_CUDA_CONT(packed, at::kInt);
    TORCH_CHECK(packed.dim() == 2 && packed.size(1) == (cols + 31) / 32, "packed must be [rows, ceil(cols/32)]");
    const int so = order_code(src_method), dso = order_code(dst_method);
    c10::cuda::CUDAGuard guard(packed.device());
    auto out = at::empty_like(packed);
    if (packed.numel() == 0) return out;
    NQ_TORCH_CHECK(nq_repack_signs(packed.data_ptr<int32_t>(), packed.size(0), cols, so, dso, out.data_ptr<int32_t>(),
                                   cur_stream(packed)));
    return out;
}

at::Tensor repack_signs_meta(const at::Tensor &packed, int64_t, const std::string &, const std::string &) {
    return at::empty_like(packed);
}

at::Tensor gemv_cuda(const at::Tensor &x, const at::Tensor &s2, const at::Tensor &vbits,
                     const std::optional<at::Tensor> &smid, const at::Tensor &ubits, const at::Tensor &s1) {
    auto a = check_layer(x, s2, vbits, smid, ubits, s1);
    at::Tensor y = run_gemv(a);
    return x.dim() == 1 ? y.squeeze(0) : y;
}

at::Tensor gemm_cuda(const at::Tensor &x, const at::Tensor &s2, const at::Tensor &vbits,
                     const std::optional<at::Tensor> &smid, const at::Tensor &ubits, const at::Tensor &s1,
                     bool precise) {
    auto a = check_layer(x, s2, vbits, smid, ubits, s1);
    at::Tensor y = run_gemm(a, precise);
    return x.dim() == 1 ? y.squeeze(0) : y;
}

at::Tensor linear_cuda(const at::Tensor &x, const at::Tensor &s2, const at::Tensor &vbits,
                       const std::optional<at::Tensor> &smid, const at::Tensor &ubits, const at::Tensor &s1) {
    return forward_auto(check_layer(x, s2, vbits, smid, ubits, s1));
}

at::Tensor layer_meta(const at::Tensor &x, const at::Tensor &, const at::Tensor &, const std::optional<at::Tensor> &,
                      const at::Tensor &, const at::Tensor &s1) {
    auto shape = x.sizes().vec();
    shape.back() = s1.numel();
    return at::empty(shape, x.options());
}

at::Tensor gemm_meta(const at::Tensor &x, const at::Tensor &s2, const at::Tensor &v, const std::optional<at::Tensor> &m,
                     const at::Tensor &u, const at::Tensor &s1, bool) {
    return layer_meta(x, s2, v, m, u, s1);
}


// ------------------------------------------------------------------ decoder-step kernels

std::tuple<at::Tensor, at::Tensor> rmsnorm_cuda(const at::Tensor &x, const std::optional<at::Tensor> &residual,
                                                const at::Tensor &weight, double eps) {
    const auto st = x.scalar_type();
    CHECK_CUDA_CONT(x, st);
    CHECK_CUDA_CONT(weight, st);
    const int64_t hidden = x.size(-1), rows = x.numel() / hidden;
    TORCH_CHECK(weight.numel() == hidden, "weight size mismatch");
    c10::cuda::CUDAGuard guard(x.device());
    auto out = at::empty_like(x);
    auto res_out = at::empty_like(x);
    const void *rin = nullptr;
    if (residual.has_value() && residual->defined()) {
        CHECK_CUDA_CONT((*residual), st);
        TORCH_CHECK(residual->numel() == x.numel(), "residual size mismatch");
        rin = residual->data_ptr();
    }
    NQ_TORCH_CHECK(nq_rmsnorm(dtype_code(st), x.data_ptr(), rin, res_out.data_ptr(), weight.data_ptr(),
                              out.data_ptr(), rows, hidden, (float)eps, cur_stream(x)));
    return {out, res_out};
}

std::tuple<at::Tensor, at::Tensor> rmsnorm_meta(const at::Tensor &x, const std::optional<at::Tensor> &,
                                                const at::Tensor &, double) {
    return {at::empty_like(x), at::empty_like(x)};
}

void rope_cache_cuda(at::Tensor &q, at::Tensor &k, const at::Tensor &v, const at::Tensor &positions,
                     const std::optional<at::Tensor> &batch_of, at::Tensor &k_cache, at::Tensor &v_cache,
                     double theta) {
    const auto st = q.scalar_type();
    CHECK_CUDA_CONT(q, st);
    CHECK_CUDA_CONT(k, st);
    CHECK_CUDA_CONT(v, st);
    CHECK_CUDA_CONT(k_cache, st);
    CHECK_CUDA_CONT(v_cache, st);
    CHECK_CUDA_CONT(positions, at::kInt);
    TORCH_CHECK(q.dim() == 3 && k.dim() == 3 && v.sizes() == k.sizes(), "q [n, hq, d], k/v [n, hkv, d]");
    TORCH_CHECK(k_cache.dim() == 4 && k_cache.sizes() == v_cache.sizes(), "caches [batch, hkv, max_seq, d]");
    const int64_t n = q.size(0), hq = q.size(1), d = q.size(2), hkv = k.size(1);
    TORCH_CHECK(k.size(0) == n && k.size(2) == d && k_cache.size(1) == hkv && k_cache.size(3) == d, "shape mismatch");
    TORCH_CHECK(positions.numel() == n, "one position per token row");
    const int32_t *bo = nullptr;
    if (batch_of.has_value() && batch_of->defined()) {
        CHECK_CUDA_CONT((*batch_of), at::kInt);
        TORCH_CHECK(batch_of->numel() == n, "one batch index per token row");
        bo = batch_of->data_ptr<int32_t>();
    } else {
        TORCH_CHECK(n <= k_cache.size(0), "without batch_of, token row t writes cache row t");
    }
    c10::cuda::CUDAGuard guard(q.device());
    NQ_TORCH_CHECK(nq_rope_cache(dtype_code(st), q.data_ptr(), k.data_ptr(), v.data_ptr(), positions.data_ptr<int32_t>(),
                                 bo, k_cache.data_ptr(), v_cache.data_ptr(), n, hq, hkv, d, k_cache.size(2),
                                 (float)theta, cur_stream(q)));
}

void rope_cache_meta(at::Tensor &, at::Tensor &, const at::Tensor &, const at::Tensor &,
                     const std::optional<at::Tensor> &, at::Tensor &, at::Tensor &, double) {}

at::Tensor decode_attention_cuda(const at::Tensor &q, const at::Tensor &k_cache, const at::Tensor &v_cache,
                                 const at::Tensor &seq_len) {
    const auto st = q.scalar_type();
    CHECK_CUDA_CONT(q, st);
    CHECK_CUDA_CONT(k_cache, st);
    CHECK_CUDA_CONT(v_cache, st);
    CHECK_CUDA_CONT(seq_len, at::kInt);
    TORCH_CHECK(q.dim() == 3 && k_cache.dim() == 4, "q [batch, hq, d], caches [batch, hkv, max_seq, d]");
    const int64_t b = q.size(0), hq = q.size(1), d = q.size(2), hkv = k_cache.size(1), ms = k_cache.size(2);
    TORCH_CHECK(k_cache.size(0) >= b && seq_len.numel() == b, "batch mismatch");
    c10::cuda::CUDAGuard guard(q.device());
    auto out = at::empty_like(q);
    const size_t wsb = nq_decode_attention_workspace_bytes(b, hq, d, ms);
    at::Tensor ws = workspace_for(q, wsb, 1);
    NQ_TORCH_CHECK(nq_decode_attention(dtype_code(st), q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                                       seq_len.data_ptr<int32_t>(), out.data_ptr(), b, hq, hkv, d, ms, ws.data_ptr(),
                                       (size_t)ws.numel(), cur_stream(q)));
    return out;
}

at::Tensor decode_attention_rope_cuda(const at::Tensor &q, const at::Tensor &k, const at::Tensor &v,
                                      const at::Tensor &positions, at::Tensor &k_cache, at::Tensor &v_cache,
                                      double theta) {
    const auto st = q.scalar_type();
    CHECK_CUDA_CONT(q, st);
    CHECK_CUDA_CONT(k, st);
    CHECK_CUDA_CONT(v, st);
    CHECK_CUDA_CONT(k_cache, st);
    CHECK_CUDA_CONT(v_cache, st);
    CHECK_CUDA_CONT(positions, at::kInt);
    TORCH_CHECK(q.dim() == 3 && k.dim() == 3 && v.sizes() == k.sizes(), "q [batch, hq, d], k/v [batch, hkv, d]");
    TORCH_CHECK(k_cache.dim() == 4 && k_cache.sizes() == v_cache.sizes(), "caches [batch, hkv, max_seq, d]");
    const int64_t b = q.size(0), hq = q.size(1), d = q.size(2), hkv = k.size(1), ms = k_cache.size(2);
    TORCH_CHECK(k.size(0) == b && k.size(2) == d && k_cache.size(1) == hkv && k_cache.size(3) == d, "shape mismatch");
    TORCH_CHECK(k_cache.size(0) >= b && positions.numel() == b, "one position per batch row");
    c10::cuda::CUDAGuard guard(q.device());
    auto out = at::empty_like(q);
    const size_t wsb = nq_decode_attention_workspace_bytes(b, hq, d, ms);
    at::Tensor ws = workspace_for(q, wsb, 1);
    NQ_TORCH_CHECK(nq_decode_attention_rope(dtype_code(st), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                            positions.data_ptr<int32_t>(), k_cache.data_ptr(), v_cache.data_ptr(),
                                            out.data_ptr(), b, hq, hkv, d, ms, (float)theta, ws.data_ptr(),
                                            (size_t)ws.numel(), cur_stream(q)));
    return out;
}

at::Tensor decode_attention_rope_meta(const at::Tensor &q, const at::Tensor &, const at::Tensor &, const at::Tensor &,
                                      at::Tensor &, at::Tensor &, double) {
    return at::empty_like(q);
}

at::Tensor decode_attention_meta(const at::Tensor &q, const at::Tensor &, const at::Tensor &, const at::Tensor &) {
    return at::empty_like(q);
}

at::Tensor silu_mul_cuda(const at::Tensor &gate, const at::Tensor &up) {
    const auto st = gate.scalar_type();
    CHECK_CUDA_CONT(gate, st);
    CHECK_CUDA_CONT(up, st);
    TORCH_CHECK(gate.sizes() == up.sizes(), "gate and up must have the same shape");
    c10::cuda::CUDAGuard guard(gate.device());
    auto out = at::empty_like(gate);
    NQ_TORCH_CHECK(nq_silu_mul(dtype_code(st), gate.data_ptr(), up.data_ptr(), out.data_ptr(), gate.numel(),
                               cur_stream(gate)));
    return out;
}

at::Tensor silu_mul_meta(const at::Tensor &gate, const at::Tensor &) { return at::empty_like(gate); }


// ------------------------------------------------------------------ grouped layers sharing one input

std::vector<at::Tensor> run_group(const at::Tensor &x, const std::vector<LayerArgs> &ls) {
    c10::cuda::CUDAGuard guard(x.device());
    std::vector<nq_gemv_layer> desc(ls.size());
    std::vector<int64_t> ranks(ls.size());
    std::vector<at::Tensor> ys;
    for (size_t i = 0; i < ls.size(); ++i) {
        const LayerArgs &a = ls[i];
        ys.push_back(at::empty({a.rows, a.out_f}, x.options()));
        desc[i].scale_pre = a.s2.data_ptr();
        desc[i].v_bits = a.vbits.data_ptr<int32_t>();
        desc[i].rank = a.rank;
        desc[i].scale_mid = a.smid ? a.smid->data_ptr() : nullptr;
        desc[i].u_bits = a.ubits.data_ptr<int32_t>();
        desc[i].out_features = a.out_f;
        desc[i].scale_post = a.s1.data_ptr();
        desc[i].y = ys.back().data_ptr();
        ranks[i] = a.rank;
    }
    const size_t wsb = nq_gemv_group_workspace_bytes((int)ls.size(), ranks.data());
    at::Tensor ws = workspace_for(x, wsb);
    NQ_TORCH_CHECK(nq_gemv_group(dtype_code(x.scalar_type()), x.data_ptr(), ls[0].rows, ls[0].in_f, (int)ls.size(),
                                 desc.data(), ws.data_ptr(), (size_t)ws.numel(), cur_stream(x)));
    return ys;
}

// Grouped GEMV on x' formed in the prologue (RMSNorm with residual, SiLU*up, x*up) with optional
// SiLU on chosen outputs: one launch for what the decoder otherwise runs as 2-3.
std::vector<at::Tensor> run_group_ex(const at::Tensor &x, const std::vector<LayerArgs> &ls, int64_t x_mode,
                                     const std::optional<at::Tensor> &x2, const std::optional<at::Tensor> &nw,
                                     double eps, const std::optional<at::Tensor> &res_out, int64_t act,
                                     const nq_tp_exchange *tp = nullptr, int tp_mode = 0) {
    c10::cuda::CUDAGuard guard(x.device());
    const auto st = x.scalar_type();
    nq_gemv_input in{};
    in.x_mode = (int)x_mode;
    in.eps = (float)eps;
    in.x = x.data_ptr();
    if (x2.has_value() && x2->defined()) {
        CHECK_CUDA_CONT((*x2), st);
        TORCH_CHECK(x2->numel() == x.numel(), "x2 must have the shape of x");
        in.x2 = x2->data_ptr();
    }
    if (nw.has_value() && nw->defined()) {
        CHECK_CUDA_CONT((*nw), st);
        TORCH_CHECK(nw->numel() == ls[0].in_f, "norm_weight must have in_features values");
        in.norm_weight = nw->data_ptr();
    }
    if (res_out.has_value() && res_out->defined()) {
        CHECK_CUDA_CONT((*res_out), st);
        TORCH_CHECK(res_out->numel() == x.numel(), "residual_out must have the shape of x");
        in.residual_out = res_out->data_ptr();
    }
    std::vector<nq_gemv_layer> desc(ls.size());
    std::vector<int64_t> ranks(ls.size());
    std::vector<at::Tensor> ys;
    for (size_t i = 0; i < ls.size(); ++i) {
        const LayerArgs &a = ls[i];
        ys.push_back(at::empty({a.rows, a.out_f}, x.options()));
        desc[i].scale_pre = a.s2.data_ptr();
        desc[i].v_bits = a.vbits.data_ptr<int32_t>();
        desc[i].rank = a.rank;
        desc[i].scale_mid = a.smid ? a.smid->data_ptr() : nullptr;
        desc[i].u_bits = a.ubits.data_ptr<int32_t>();
        desc[i].out_features = a.out_f;
        desc[i].scale_post = a.s1.data_ptr();
        desc[i].y = ys.back().data_ptr();
        ranks[i] = a.rank;
    }
    const size_t wsb = nq_gemv_group_workspace_bytes((int)ls.size(), ranks.data());
    at::Tensor ws = workspace_for(x, wsb);
    if (tp_mode)
        NQ_TORCH_CHECK(nq_gemv_group_tp(dtype_code(st), &in, ls[0].rows, ls[0].in_f, (int)ls.size(), desc.data(),
                                        (int)act, tp, tp_mode, ws.data_ptr(), (size_t)ws.numel(), cur_stream(x)));
    else
        NQ_TORCH_CHECK(nq_gemv_group_ex(dtype_code(st), &in, ls[0].rows, ls[0].in_f, (int)ls.size(), desc.data(),
                                        (int)act, ws.data_ptr(), (size_t)ws.numel(), cur_stream(x)));
    return ys;
}

nq_tp_exchange make_exchange(at::IntArrayRef regions, int64_t rank, int64_t max_elems) {
    TORCH_CHECK(regions.size() >= 1 && regions.size() <= 8, "1..8 exchange regions");
    nq_tp_exchange x{};
    for (size_t r = 0; r < regions.size(); ++r) x.regions[r] = reinterpret_cast<void *>(regions[r]);
    x.rank = (int)rank;
    x.world = (int)regions.size();
    x.max_elems = max_elems;
    return x;
}

std::vector<LayerArgs> check_group(const at::Tensor &x, const std::vector<at::Tensor> &s2,
                                   const std::vector<at::Tensor> &vbits,
                                   const std::vector<std::optional<at::Tensor>> &smid,
                                   const std::vector<at::Tensor> &ubits, const std::vector<at::Tensor> &s1) {
    const size_t n = s2.size();
    TORCH_CHECK(n >= 1 && n <= 3, "a layer group holds 1 to 3 layers");
    TORCH_CHECK(vbits.size() == n && smid.size() == n && ubits.size() == n && s1.size() == n,
                "every per-layer list must have the same length");
    std::vector<LayerArgs> ls;
    for (size_t i = 0; i < n; ++i) ls.push_back(check_layer(x, s2[i], vbits[i], smid[i], ubits[i], s1[i]));
    return ls;
}

std::vector<at::Tensor> gemv_group_cuda(const at::Tensor &x, at::TensorList s2, at::TensorList vbits,
                                        const c10::List<std::optional<at::Tensor>> &smid, at::TensorList ubits,
                                        at::TensorList s1) {
    std::vector<std::optional<at::Tensor>> sm(smid.begin(), smid.end());
    auto ls = check_group(x, s2.vec(), vbits.vec(), sm, ubits.vec(), s1.vec());
    auto ys = run_group(x, ls);
    if (x.dim() == 1)
        for (auto &y : ys) y = y.squeeze(0);
    return ys;
}

std::vector<at::Tensor> gemv_group_tp_cuda(const at::Tensor &x, const std::optional<at::Tensor> &x2,
                                           const std::optional<at::Tensor> &norm_weight, double eps, int64_t x_mode,
                                           const std::optional<at::Tensor> &residual_out, int64_t act,
                                           at::TensorList s2, at::TensorList vbits,
                                           const c10::List<std::optional<at::Tensor>> &smid, at::TensorList ubits,
                                           at::TensorList s1, at::IntArrayRef regions, int64_t rank,
                                           int64_t max_elems, int64_t tp_mode) {
    std::vector<std::optional<at::Tensor>> sm(smid.begin(), smid.end());
    auto ls = check_group(x, s2.vec(), vbits.vec(), sm, ubits.vec(), s1.vec());
    const nq_tp_exchange ex = make_exchange(regions, rank, max_elems);
    auto ys = run_group_ex(x, ls, x_mode, x2, norm_weight, eps, residual_out, act, &ex, (int)tp_mode);
    if (x.dim() == 1)
        for (auto &y : ys) y = y.squeeze(0);
    return ys;
}

at::Tensor tp_pull_cuda(const at::Tensor &like, at::IntArrayRef regions, int64_t rank, int64_t max_elems) {
    CHECK_CUDA_CONT(like, like.scalar_type());
    c10::cuda::CUDAGuard guard(like.device());
    auto out = at::empty_like(like);
    const nq_tp_exchange ex = make_exchange(regions, rank, max_elems);
    NQ_TORCH_CHECK(nq_tp_pull(dtype_code(like.scalar_type()), &ex, like.numel(), out.data_ptr(), cur_stream(like)));
    return out;
}

std::vector<at::Tensor> gemv_group_ex_cuda(const at::Tensor &x, const std::optional<at::Tensor> &x2,
                                           const std::optional<at::Tensor> &norm_weight, double eps, int64_t x_mode,
                                           const std::optional<at::Tensor> &residual_out, int64_t act,
                                           at::TensorList s2, at::TensorList vbits,
                                           const c10::List<std::optional<at::Tensor>> &smid, at::TensorList ubits,
                                           at::TensorList s1) {
    std::vector<std::optional<at::Tensor>> sm(smid.begin(), smid.end());
    auto ls = check_group(x, s2.vec(), vbits.vec(), sm, ubits.vec(), s1.vec());
    auto ys = run_group_ex(x, ls, x_mode, x2, norm_weight, eps, residual_out, act);
    if (x.dim() == 1)
        for (auto &y : ys) y = y.squeeze(0);
    return ys;
}

std::vector<at::Tensor> group_ex_meta(const at::Tensor &x, const std::optional<at::Tensor> &,
                                      const std::optional<at::Tensor> &, double, int64_t, const std::optional<at::Tensor> &,
                                      int64_t, at::TensorList, at::TensorList, const c10::List<std::optional<at::Tensor>> &,
                                      at::TensorList, at::TensorList s1) {
    std::vector<at::Tensor> ys;
    for (const auto &s : s1) {
        auto shape = x.sizes().vec();
        shape.back() = s.numel();
        ys.push_back(at::empty(shape, x.options()));
    }
    return ys;
}

std::vector<at::Tensor> linear_group_cuda(const at::Tensor &x, at::TensorList s2, at::TensorList vbits,
                                          const c10::List<std::optional<at::Tensor>> &smid, at::TensorList ubits,
                                          at::TensorList s1) {
    std::vector<std::optional<at::Tensor>> sm(smid.begin(), smid.end());
    auto ls = check_group(x, s2.vec(), vbits.vec(), sm, ubits.vec(), s1.vec());
    std::vector<at::Tensor> ys;
    if (gemm_ok(ls[0])) {
        for (auto &a : ls) ys.push_back(run_gemm(a, true));
    } else {
        ys = run_group(x, ls);
    }
    if (x.dim() == 1)
        for (auto &y : ys) y = y.squeeze(0);
    return ys;
}

std::vector<at::Tensor> group_meta(const at::Tensor &x, at::TensorList, at::TensorList,
                                   const c10::List<std::optional<at::Tensor>> &, at::TensorList, at::TensorList s1) {
    std::vector<at::Tensor> ys;
    for (const auto &s : s1) {
        auto shape = x.sizes().vec();
        shape.back() = s.numel();
        ys.push_back(at::empty(shape, x.options()));
    }
    return ys;
}

}  // namespace

TORCH_LIBRARY(binary_kernels, m) {
    m.def(
        "nanoquant_dyn_forward("
        "Tensor x, Tensor scale_g, Tensor Ubits, Tensor? scale_l, Tensor Vbits, Tensor scale_h, "
        "int num_thread_stage1=128, int num_thread_stage2=128, int num_row_per_warp_stage1=2, "
        "int num_row_per_warp_stage2=2, int num_acc_stage1=4, int num_acc_stage2=4, "
        "int num_pipeline_stage1=2, int num_pipeline_stage2=2) -> Tensor");
    m.def(
        "marlin_onebit_forward("
        "Tensor x, Tensor weight, Tensor? scale_g, Tensor? scale_h, Tensor(a!) workspace) -> Tensor");
    m.def(
        "marlin_nanoquant_forward("
        "Tensor x, Tensor weight_u, Tensor weight_v, Tensor? scale_g, Tensor? scale_l, Tensor? scale_h, "
        "Tensor(a!) workspace) -> Tensor");
}

TORCH_LIBRARY_IMPL(binary_kernels, CUDA, m) {
    m.impl("nanoquant_dyn_forward", &nanoquant_dyn_forward_cuda);
    m.impl("marlin_onebit_forward", &marlin_onebit_forward_cuda);
    m.impl("marlin_nanoquant_forward", &marlin_nanoquant_forward_cuda);
}

TORCH_LIBRARY_IMPL(binary_kernels, Meta, m) {
    m.impl("nanoquant_dyn_forward", &nanoquant_dyn_forward_meta);
    m.impl("marlin_onebit_forward", &marlin_onebit_forward_meta);
    m.impl("marlin_nanoquant_forward", &marlin_nanoquant_forward_meta);
}

TORCH_LIBRARY(nq_b200, m) {
    m.def("pack_signs(Tensor signs, str method='lsb_first', bool check=False) -> Tensor");
    m.def("unpack_signs(Tensor packed, int rows, int cols, str method='lsb_first') -> Tensor");
    m.def("repack_signs(Tensor packed, int cols, str src_method, str dst_method) -> Tensor");
    m.def("pack_marlin(Tensor signs, bool check=False) -> Tensor");
    m.def("unpack_marlin(Tensor words, int n_out, int k_red) -> Tensor");
    m.def("marlin_to_half2(Tensor words, int n_out, int k_red) -> Tensor");
    m.def(
        "gemv(Tensor x, Tensor scale_pre, Tensor v_bits, Tensor? scale_mid, Tensor u_bits, Tensor scale_post) -> "
        "Tensor");
    m.def(
        "gemm(Tensor x, Tensor scale_pre, Tensor v_bits, Tensor? scale_mid, Tensor u_bits, Tensor scale_post, "
        "bool precise=True) -> Tensor");
    m.def(
        "linear(Tensor x, Tensor scale_pre, Tensor v_bits, Tensor? scale_mid, Tensor u_bits, Tensor scale_post) -> "
        "Tensor");
    m.def("rmsnorm(Tensor x, Tensor? residual, Tensor weight, float eps) -> (Tensor, Tensor)");
    m.def(
        "rope_cache(Tensor(a!) q, Tensor(b!) k, Tensor v, Tensor positions, Tensor? batch_of, Tensor(c!) k_cache, "
        "Tensor(d!) v_cache, float theta) -> ()");
    m.def("decode_attention(Tensor q, Tensor k_cache, Tensor v_cache, Tensor seq_len) -> Tensor");
    m.def("decode_attention_rope(Tensor q, Tensor k, Tensor v, Tensor positions, Tensor(a!) k_cache, "
          "Tensor(b!) v_cache, float theta) -> Tensor");
    m.def("silu_mul(Tensor gate, Tensor up) -> Tensor");
    m.def(
        "gemv_group(Tensor x, Tensor[] scale_pre, Tensor[] v_bits, Tensor?[] scale_mid, Tensor[] u_bits, "
        "Tensor[] scale_post) -> Tensor[]");
    m.def(
        "linear_group(Tensor x, Tensor[] scale_pre, Tensor[] v_bits, Tensor?[] scale_mid, Tensor[] u_bits, "
        "Tensor[] scale_post) -> Tensor[]");
    m.def(
        "gemv_group_ex(Tensor x, Tensor? x2, Tensor? norm_weight, float eps, int x_mode, Tensor(a!)? residual_out, "
        "int act, Tensor[] scale_pre, Tensor[] v_bits, Tensor?[] scale_mid, Tensor[] u_bits, Tensor[] scale_post) "
        "-> Tensor[]");
    m.def(
        "gemv_group_tp(Tensor x, Tensor? x2, Tensor? norm_weight, float eps, int x_mode, Tensor(a!)? residual_out, "
        "int act, Tensor[] scale_pre, Tensor[] v_bits, Tensor?[] scale_mid, Tensor[] u_bits, Tensor[] scale_post, "
        "int[] regions, int rank, int max_elems, int tp_mode) -> Tensor[]");
    m.def("tp_pull(Tensor like, int[] regions, int rank, int max_elems) -> Tensor");
}

TORCH_LIBRARY_IMPL(nq_b200, CUDA, m) {
    m.impl("pack_signs", &pack_signs_cuda);
    m.impl("unpack_signs", &unpack_signs_cuda);
    m.impl("repack_signs", &repack_signs_cuda);
    m.impl("pack_marlin", &pack_marlin_cuda);
    m.impl("unpack_marlin", &unpack_marlin_cuda);
    m.impl("marlin_to_half2", &marlin_to_half2_cuda);
    m.impl("gemv", &gemv_cuda);
    m.impl("gemm", &gemm_cuda);
    m.impl("linear", &linear_cuda);
    m.impl("rmsnorm", &rmsnorm_cuda);
    m.impl("rope_cache", &rope_cache_cuda);
    m.impl("decode_attention", &decode_attention_cuda);
    m.impl("decode_attention_rope", &decode_attention_rope_cuda);
    m.impl("silu_mul", &silu_mul_cuda);
    m.impl("gemv_group", &gemv_group_cuda);
    m.impl("gemv_group_ex", &gemv_group_ex_cuda);
    m.impl("gemv_group_tp", &gemv_group_tp_cuda);
    m.impl("tp_pull", &tp_pull_cuda);
    m.impl("linear_group", &linear_group_cuda);
}

TORCH_LIBRARY_IMPL(nq_b200, Meta, m) {
    m.impl("pack_signs", &pack_signs_meta);
    m.impl("unpack_signs", &unpack_signs_meta);
    m.impl("repack_signs", &repack_signs_meta);
    m.impl("pack_marlin", &pack_marlin_meta);
    m.impl("unpack_marlin", &unpack_marlin_meta);
    m.impl("marlin_to_half2", &marlin_to_half2_meta);
    m.impl("gemv", &layer_meta);
    m.impl("gemm", &gemm_meta);
    m.impl("linear", &layer_meta);
    m.impl("rmsnorm", &rmsnorm_meta);
    m.impl("rope_cache", &rope_cache_meta);
    m.impl("decode_attention", &decode_attention_meta);
    m.impl("decode_attention_rope", &decode_attention_rope_meta);
    m.impl("silu_mul", &silu_mul_meta);
    m.impl("gemv_group", &group_meta);
    m.impl("gemv_group_ex", &group_ex_meta);
    m.impl("linear_group", &group_meta);
}
