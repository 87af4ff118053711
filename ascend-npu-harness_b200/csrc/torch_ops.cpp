// torch custom-op registration of the ten ladder operators (namespace `hc`).
//
// A thin layer over the C ABI in include/hc_ops.h: each CUDA kernel checks its tensors, sets the
// device, allocates the outputs, launches on the current CUDA stream and turns a non-zero status
// into a torch error carrying hc_last_error_string().  The Meta kernels give output shapes
// without touching a device (fake tensors, tracing).  Nothing here computes; there is no CPU
// kernel, so a CPU tensor raises torch's "no kernel for CPU" dispatch error instead of a silent
// fallback.
//
// The schemas follow the reference runners' argument lists (ops/<op>/runner/*.hpp) with torch
// tensors in place of host pointers and shapes:
//   hc::elementwise_add(x, y)                                   elementwise_add_runner.hpp
//   hc::axpy_scalar_affine(x, alpha, beta)                      axpy_scalar_affine_runner.hpp
//   hc::broadcast_binary(x, y, bias, y_batch)                   broadcast_binary_runner.hpp
//   hc::activation_gelu_silu(x, act)       act 0 GELU, 1 SiLU   activation_gelu_silu_runner.hpp
//   hc::reduce_sum_lastdim(x)              fp32 output          reduce_sum_lastdim_runner.hpp
//   hc::transpose_2d_4d(x, mode)           0 2D, 1 NCHW->NHWC, 2 NHWC->NCHW
//   hc::layer_norm(x, gamma, beta, eps)                         layer_norm_runner.hpp
//   hc::rms_norm_rope_fused(x, weight, cos, sin, rotary_dim, eps, heads, rope_style)
//   hc::matmul_bias(a, b, bias?)                                matmul_bias_runner.hpp
//   hc::flash_attention_fwd_fused(q, k, v, scale, mask_type) -> (o, lse)   (k, v may have fewer heads: GQA)
//   hc::flash_attention_bwd(q, k, v, o, lse, dout, scale, mask_type) -> (dq, dk, dv, delta)
//                                          (no reference counterpart; K/V with the query head count)
// hc.load_torch_ops() also registers the backward as the autograd formula of the forward op.
// Load with torch.ops.load_library("ascend-npu-harness_b200/lib/libhc_torch.so").
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <cmath>
#include <optional>

#include "hc_ops.h"
#include "hc_runtime.h"

namespace {

int dtype_code(const at::Tensor& t) {
    switch (t.scalar_type()) {
        case at::kFloat: return HC_DTYPE_F32;
        case at::kHalf: return HC_DTYPE_F16;
        case at::kBFloat16: return HC_DTYPE_BF16;
        case at::kInt: return HC_DTYPE_I32;
        case at::kChar: return HC_DTYPE_I8;
        case at::kByte: return HC_DTYPE_U8;
        default: TORCH_CHECK(false, "hc: dtype ", t.scalar_type(), " is not supported");
    }
    return -1;
}

void check_input(const at::Tensor& t, const char* what) {
    TORCH_CHECK(t.is_cuda(), "hc: ", what, " must be a CUDA tensor");
    TORCH_CHECK(t.is_contiguous(), "hc: ", what, " must be contiguous");
}

void check_f32(const at::Tensor& t, const char* what, const at::Tensor& like) {
    check_input(t, what);
    TORCH_CHECK(t.scalar_type() == at::kFloat, "hc: ", what, " must be float32");
    TORCH_CHECK(t.device() == like.device(), "hc: ", what, " is on another device");
}

void* stream_of(const at::Tensor& t) {
    return static_cast<void*>(c10::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

void ok_or_throw(int status, const char* op) {
    TORCH_CHECK(status == HC_OK, "hc::", op, " failed (status ", status, "): ", hc_last_error_string());
}

uint32_t u32(int64_t v, const char* what) {
    TORCH_CHECK(v >= 0 && v <= 0xFFFFFFFFll, "hc: ", what, " = ", v, " does not fit 32 bits");
    return static_cast<uint32_t>(v);
}

// ---------------------------------------------------------------------------------------------
// CUDA kernels
// ---------------------------------------------------------------------------------------------
at::Tensor elementwise_add_cuda(const at::Tensor& x, const at::Tensor& y) {
    check_input(x, "x");
    check_input(y, "y");
    TORCH_CHECK(x.sizes() == y.sizes() && x.scalar_type() == y.scalar_type(), "hc: x and y differ in shape or dtype");
    c10::cuda::CUDAGuard guard(x.device());
    at::Tensor z = at::empty_like(x);
    elementwise_add_tiling_data t{u32(x.numel(), "numel"), 0};
    ok_or_throw(hc_elementwise_add_launch(x.data_ptr(), y.data_ptr(), z.data_ptr(), &t, dtype_code(x), stream_of(x)),
                "elementwise_add");
    return z;
}

at::Tensor axpy_scalar_affine_cuda(const at::Tensor& x, double alpha, double beta) {
    check_input(x, "x");
    c10::cuda::CUDAGuard guard(x.device());
    at::Tensor y = at::empty_like(x);
    axpy_scalar_affine_tiling_data t{u32(x.numel(), "numel"), 0};
    ok_or_throw(hc_axpy_scalar_affine_launch(x.data_ptr(), y.data_ptr(), &t, static_cast<float>(alpha),
                                             static_cast<float>(beta), dtype_code(x), stream_of(x)),
                "axpy_scalar_affine");
    return y;
}

at::Tensor broadcast_binary_cuda(const at::Tensor& x, const at::Tensor& y, const at::Tensor& bias, int64_t y_batch) {
    check_input(x, "x");
    check_input(y, "y");
    check_input(bias, "bias");
    TORCH_CHECK(x.dim() == 4, "hc: broadcast_binary x must be NCHW");
    TORCH_CHECK(y.scalar_type() == x.scalar_type() && bias.scalar_type() == x.scalar_type(),
                "hc: broadcast_binary x, y and bias must share a dtype");
    TORCH_CHECK(y.numel() == y_batch * x.size(1) && bias.numel() == x.size(1),
                "hc: broadcast_binary expects y of y_batch x C and bias of C elements");
    c10::cuda::CUDAGuard guard(x.device());
    at::Tensor z = at::empty_like(x);
    broadcast_binary_tiling_data t{u32(x.size(0), "B"), u32(x.size(1), "C"), u32(x.size(2), "H"), u32(x.size(3), "W"),
                                   u32(y_batch, "y_batch"), 0};
    ok_or_throw(hc_broadcast_binary_launch(x.data_ptr(), y.data_ptr(), bias.data_ptr(), z.data_ptr(), &t,
                                           dtype_code(x), stream_of(x)),
                "broadcast_binary");
    return z;
}

at::Tensor activation_gelu_silu_cuda(const at::Tensor& x, int64_t act) {
    check_input(x, "x");
    c10::cuda::CUDAGuard guard(x.device());
    at::Tensor y = at::empty_like(x);
    activation_gelu_silu_tiling_data t{u32(x.numel(), "numel"), 0, u32(act, "act")};
    ok_or_throw(hc_activation_gelu_silu_launch(x.data_ptr(), y.data_ptr(), &t, dtype_code(x), stream_of(x)),
                "activation_gelu_silu");
    return y;
}

at::Tensor reduce_sum_lastdim_cuda(const at::Tensor& x) {
    check_input(x, "x");
    TORCH_CHECK(x.dim() >= 1, "hc: reduce_sum_lastdim needs at least one dimension");
    c10::cuda::CUDAGuard guard(x.device());
    const int64_t K = x.size(-1);
    at::Tensor out = at::empty(x.sizes().slice(0, x.dim() - 1), x.options().dtype(at::kFloat));
    reduce_sum_lastdim_tiling_data t{u32(K ? x.numel() / K : 0, "rows"), u32(K, "K"), 0};
    ok_or_throw(hc_reduce_sum_lastdim_launch(x.data_ptr(), out.data_ptr<float>(), &t, dtype_code(x), stream_of(x)),
                "reduce_sum_lastdim");
    return out;
}

std::vector<int64_t> transpose_shape(const at::Tensor& x, int64_t mode, transpose_2d_4d_tiling_data* t) {
    if (mode == 0) {
        TORCH_CHECK(x.dim() == 2, "hc: transpose_2d_4d mode 0 needs a 2-D tensor");
        if (t) *t = {0, u32(x.size(0), "M"), u32(x.size(1), "N"), 0, 0, 0};
        return {x.size(1), x.size(0)};
    }
    TORCH_CHECK(x.dim() == 4, "hc: transpose_2d_4d modes 1 and 2 need a 4-D tensor");
    if (mode == 1) {  // NCHW -> NHWC
        if (t) *t = {1, u32(x.size(0), "N"), u32(x.size(1), "C"), u32(x.size(2), "H"), u32(x.size(3), "W"), 0};
        return {x.size(0), x.size(2), x.size(3), x.size(1)};
    }
    TORCH_CHECK(mode == 2, "hc: transpose_2d_4d mode ", mode, " (0 = 2D, 1 = NCHW->NHWC, 2 = NHWC->NCHW)");
    if (t) *t = {2, u32(x.size(0), "N"), u32(x.size(3), "C"), u32(x.size(1), "H"), u32(x.size(2), "W"), 0};
    return {x.size(0), x.size(3), x.size(1), x.size(2)};
}

at::Tensor transpose_2d_4d_cuda(const at::Tensor& x, int64_t mode) {
    check_input(x, "x");
    transpose_2d_4d_tiling_data t{};
    const std::vector<int64_t> shape = transpose_shape(x, mode, &t);
    c10::cuda::CUDAGuard guard(x.device());
    at::Tensor out = at::empty(shape, x.options());
    ok_or_throw(hc_transpose_2d_4d_launch(x.data_ptr(), out.data_ptr(), &t, dtype_code(x), stream_of(x)),
                "transpose_2d_4d");
    return out;
}

at::Tensor layer_norm_cuda(const at::Tensor& x, const at::Tensor& gamma, const at::Tensor& beta, double eps) {
    check_input(x, "x");
    check_f32(gamma, "gamma", x);
    check_f32(beta, "beta", x);
    TORCH_CHECK(x.dim() >= 1 && gamma.numel() == x.size(-1) && beta.numel() == x.size(-1),
                "hc: layer_norm gamma and beta need last_dim elements");
    c10::cuda::CUDAGuard guard(x.device());
    at::Tensor y = at::empty_like(x);
    const int64_t last = x.size(-1);
    layer_norm_tiling_data t{u32(last ? x.numel() / last : 0, "rows"), u32(last, "last_dim"), 0,
                             static_cast<float>(eps)};
    ok_or_throw(hc_layer_norm_launch(x.data_ptr(), gamma.data_ptr<float>(), beta.data_ptr<float>(), y.data_ptr(), &t,
                                     dtype_code(x), stream_of(x)),
                "layer_norm");
    return y;
}

at::Tensor rms_norm_rope_fused_cuda(const at::Tensor& x, const at::Tensor& weight, const at::Tensor& cos_t,
                                    const at::Tensor& sin_t, int64_t rotary_dim, double eps, int64_t heads,
                                    int64_t rope_style) {
    check_input(x, "x");
    check_f32(weight, "weight", x);
    check_f32(cos_t, "cos", x);
    check_f32(sin_t, "sin", x);
    TORCH_CHECK(x.dim() == 3 || x.dim() == 4, "hc: rms_norm_rope_fused x must be [B, S, H] or [B, S, heads, H]");
    TORCH_CHECK(x.dim() == 3 ? heads == 1 : heads == x.size(2), "hc: rms_norm_rope_fused heads does not match x");
    c10::cuda::CUDAGuard guard(x.device());
    at::Tensor out = at::empty_like(x);
    rms_norm_rope_fused_tiling_data t{u32(x.size(0), "B"), u32(x.size(1), "S"), u32(x.size(-1), "H"),
                                      u32(rotary_dim, "rotary_dim"), 0, static_cast<float>(eps)};
    ok_or_throw(hc_rms_norm_rope_fused_launch(x.data_ptr(), weight.data_ptr<float>(), cos_t.data_ptr<float>(),
                                              sin_t.data_ptr<float>(), out.data_ptr(), &t, u32(heads, "heads"),
                                              u32(rope_style, "rope_style"), dtype_code(x), stream_of(x)),
                "rms_norm_rope_fused");
    return out;
}

at::Tensor matmul_bias_cuda(const at::Tensor& a, const at::Tensor& b, const std::optional<at::Tensor>& bias) {
    check_input(a, "a");
    check_input(b, "b");
    TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(0), "hc: matmul_bias needs a [M, K] and b [K, N]");
    TORCH_CHECK(a.scalar_type() == b.scalar_type(), "hc: matmul_bias a and b must share a dtype");
    if (bias) {
        check_input(*bias, "bias");
        TORCH_CHECK(bias->numel() == b.size(1) && bias->scalar_type() == a.scalar_type(),
                    "hc: matmul_bias bias needs N elements of the operands' dtype");
    }
    c10::cuda::CUDAGuard guard(a.device());
    at::Tensor c = at::empty({a.size(0), b.size(1)}, a.options());
    matmul_bias_tiling_data t{u32(a.size(0), "M"), u32(a.size(1), "K"), u32(b.size(1), "N"), 0, 0, 0};
    ok_or_throw(hc_matmul_bias_launch(a.data_ptr(), b.data_ptr(), bias ? bias->data_ptr() : nullptr, c.data_ptr(), &t,
                                      dtype_code(a), stream_of(a)),
                "matmul_bias");
    return c;
}

std::tuple<at::Tensor, at::Tensor> flash_attention_fwd_fused_cuda(const at::Tensor& q, const at::Tensor& k,
                                                                  const at::Tensor& v, double scale,
                                                                  int64_t mask_type) {
    check_input(q, "q");
    check_input(k, "k");
    check_input(v, "v");
    TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "hc: flash attention tensors are [B, H, S, D]");
    TORCH_CHECK(k.size(0) == q.size(0) && v.size(0) == q.size(0) && v.size(1) == k.size(1) && k.size(3) == q.size(3) &&
                    v.size(2) == k.size(2),
                "hc: flash attention q, k, v shapes disagree");
    TORCH_CHECK(k.size(1) >= 1 && q.size(1) % k.size(1) == 0,
                "hc: flash attention K/V heads (", k.size(1), ") must divide the query heads (", q.size(1), ")");
    TORCH_CHECK(k.scalar_type() == q.scalar_type() && v.scalar_type() == q.scalar_type(),
                "hc: flash attention q, k, v must share a dtype");
    c10::cuda::CUDAGuard guard(q.device());
    at::Tensor o = at::empty({q.size(0), q.size(1), q.size(2), v.size(3)}, q.options());
    at::Tensor lse = at::empty({q.size(0), q.size(1), q.size(2)}, q.options().dtype(at::kFloat));
    flash_attention_fwd_fused_tiling_data t{u32(q.size(0), "B"), u32(q.size(1), "H"), u32(q.size(2), "S_q"),
                                            u32(k.size(2), "S_k"), u32(q.size(3), "D"), u32(v.size(3), "D_v"),
                                            static_cast<float>(scale), u32(mask_type, "mask_type")};
    ok_or_throw(hc_flash_attention_fwd_fused_gqa_launch(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                                        lse.data_ptr<float>(), &t, u32(k.size(1), "kv_heads"),
                                                        dtype_code(q), stream_of(q)),
                "flash_attention_fwd_fused");
    return {o, lse};
}

std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor> flash_attention_bwd_cuda(
    const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o, const at::Tensor& lse,
    const at::Tensor& dout, double scale, int64_t mask_type) {
    for (const auto& [t, n] : {std::pair<const at::Tensor&, const char*>{q, "q"}, {k, "k"}, {v, "v"}, {o, "o"},
                               {dout, "dout"}})
        check_input(t, n);
    check_input(lse, "lse");
    TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "hc: flash attention tensors are [B, H, S, D]");
    TORCH_CHECK(k.sizes() == at::IntArrayRef({q.size(0), q.size(1), k.size(2), q.size(3)}) && v.size(0) == q.size(0) &&
                    v.size(1) == q.size(1) && v.size(2) == k.size(2),
                "hc: flash_attention_bwd needs K/V with the query head count and matching shapes");
    TORCH_CHECK(o.sizes() == at::IntArrayRef({q.size(0), q.size(1), q.size(2), v.size(3)}) && dout.sizes() == o.sizes(),
                "hc: flash_attention_bwd o / dout shape");
    TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.sizes() == at::IntArrayRef({q.size(0), q.size(1), q.size(2)}),
                "hc: flash_attention_bwd lse must be fp32 [B, H, S_q]");
    for (const at::Tensor* t : {&k, &v, &o, &dout})
        TORCH_CHECK(t->scalar_type() == q.scalar_type(), "hc: flash_attention_bwd tensors must share a dtype");
    c10::cuda::CUDAGuard guard(q.device());
    at::Tensor dq = at::empty_like(q), dk = at::empty_like(k), dv = at::empty_like(v);
    at::Tensor delta = at::empty({q.size(0), q.size(1), q.size(2)}, q.options().dtype(at::kFloat));
    flash_attention_fwd_fused_tiling_data t{u32(q.size(0), "B"), u32(q.size(1), "H"), u32(q.size(2), "S_q"),
                                            u32(k.size(2), "S_k"), u32(q.size(3), "D"), u32(v.size(3), "D_v"),
                                            static_cast<float>(scale), u32(mask_type, "mask_type")};
    ok_or_throw(hc_flash_attention_bwd_launch(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), dout.data_ptr(),
                                              lse.data_ptr<float>(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                                              delta.data_ptr<float>(), &t, dtype_code(q), stream_of(q)),
                "flash_attention_bwd");
    return {dq, dk, dv, delta};
}

// ---------------------------------------------------------------------------------------------
// Meta kernels (shapes only)
// ---------------------------------------------------------------------------------------------
at::Tensor same_meta(const at::Tensor& x) { return at::empty_like(x); }
at::Tensor elementwise_add_meta(const at::Tensor& x, const at::Tensor&) { return same_meta(x); }
at::Tensor axpy_scalar_affine_meta(const at::Tensor& x, double, double) { return same_meta(x); }
at::Tensor broadcast_binary_meta(const at::Tensor& x, const at::Tensor&, const at::Tensor&, int64_t) {
    return same_meta(x);
}
at::Tensor activation_gelu_silu_meta(const at::Tensor& x, int64_t) { return same_meta(x); }
at::Tensor reduce_sum_lastdim_meta(const at::Tensor& x) {
    return at::empty(x.sizes().slice(0, x.dim() - 1), x.options().dtype(at::kFloat));
}
at::Tensor transpose_2d_4d_meta(const at::Tensor& x, int64_t mode) {
    return at::empty(transpose_shape(x, mode, nullptr), x.options());
}
at::Tensor layer_norm_meta(const at::Tensor& x, const at::Tensor&, const at::Tensor&, double) { return same_meta(x); }
at::Tensor rms_norm_rope_fused_meta(const at::Tensor& x, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                    int64_t, double, int64_t, int64_t) {
    return same_meta(x);
}
at::Tensor matmul_bias_meta(const at::Tensor& a, const at::Tensor& b, const std::optional<at::Tensor>&) {
    return at::empty({a.size(0), b.size(1)}, a.options());
}
std::tuple<at::Tensor, at::Tensor> flash_attention_fwd_fused_meta(const at::Tensor& q, const at::Tensor& k,
                                                                  const at::Tensor& v, double, int64_t) {
    TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "hc: flash attention tensors are [B, H, S, D]");
    TORCH_CHECK(k.size(1) >= 1 && q.size(1) % k.size(1) == 0,
                "hc: flash attention K/V heads (", k.size(1), ") must divide the query heads (", q.size(1), ")");
    return {at::empty({q.size(0), q.size(1), q.size(2), v.size(3)}, q.options()),
            at::empty({q.size(0), q.size(1), q.size(2)}, q.options().dtype(at::kFloat))};
}

std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor> flash_attention_bwd_meta(
    const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor&, const at::Tensor&,
    const at::Tensor&, double, int64_t) {
    return {at::empty_like(q), at::empty_like(k), at::empty_like(v),
            at::empty({q.size(0), q.size(1), q.size(2)}, q.options().dtype(at::kFloat))};
}

}  // namespace

TORCH_LIBRARY(hc, m) {
    m.def("elementwise_add(Tensor x, Tensor y) -> Tensor");
    m.def("axpy_scalar_affine(Tensor x, float alpha, float beta) -> Tensor");
    m.def("broadcast_binary(Tensor x, Tensor y, Tensor bias, int y_batch) -> Tensor");
    m.def("activation_gelu_silu(Tensor x, int act) -> Tensor");
    m.def("reduce_sum_lastdim(Tensor x) -> Tensor");
    m.def("transpose_2d_4d(Tensor x, int mode) -> Tensor");
    m.def("layer_norm(Tensor x, Tensor gamma, Tensor beta, float eps) -> Tensor");
    m.def("rms_norm_rope_fused(Tensor x, Tensor weight, Tensor cos, Tensor sin, int rotary_dim, float eps, "
          "int heads=1, int rope_style=0) -> Tensor");
    m.def("matmul_bias(Tensor a, Tensor b, Tensor? bias=None) -> Tensor");
    m.def("flash_attention_fwd_fused(Tensor q, Tensor k, Tensor v, float scale, int mask_type) -> (Tensor, Tensor)");
    m.def("flash_attention_bwd(Tensor q, Tensor k, Tensor v, Tensor o, Tensor lse, Tensor dout, float scale, "
          "int mask_type) -> (Tensor, Tensor, Tensor, Tensor)");
}

TORCH_LIBRARY_IMPL(hc, CUDA, m) {
    m.impl("elementwise_add", &elementwise_add_cuda);
    m.impl("axpy_scalar_affine", &axpy_scalar_affine_cuda);
    m.impl("broadcast_binary", &broadcast_binary_cuda);
    m.impl("activation_gelu_silu", &activation_gelu_silu_cuda);
    m.impl("reduce_sum_lastdim", &reduce_sum_lastdim_cuda);
    m.impl("transpose_2d_4d", &transpose_2d_4d_cuda);
    m.impl("layer_norm", &layer_norm_cuda);
    m.impl("rms_norm_rope_fused", &rms_norm_rope_fused_cuda);
    m.impl("matmul_bias", &matmul_bias_cuda);
    m.impl("flash_attention_fwd_fused", &flash_attention_fwd_fused_cuda);
    m.impl("flash_attention_bwd", &flash_attention_bwd_cuda);
}

TORCH_LIBRARY_IMPL(hc, Meta, m) {
    m.impl("elementwise_add", &elementwise_add_meta);
    m.impl("axpy_scalar_affine", &axpy_scalar_affine_meta);
    m.impl("broadcast_binary", &broadcast_binary_meta);
    m.impl("activation_gelu_silu", &activation_gelu_silu_meta);
    m.impl("reduce_sum_lastdim", &reduce_sum_lastdim_meta);
    m.impl("transpose_2d_4d", &transpose_2d_4d_meta);
    m.impl("layer_norm", &layer_norm_meta);
    m.impl("rms_norm_rope_fused", &rms_norm_rope_fused_meta);
    m.impl("matmul_bias", &matmul_bias_meta);
    m.impl("flash_attention_fwd_fused", &flash_attention_fwd_fused_meta);
    m.impl("flash_attention_bwd", &flash_attention_bwd_meta);
}
