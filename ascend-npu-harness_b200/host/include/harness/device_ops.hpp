// C++ runners of the ten ladder operators on B200, built on the C-ABI in hc_ops.h.
//
// The reference gives every operator a runner with host pointers (ops/<op>/runner/*.hpp): the
// elementwise family as harness::runner::<op>::run(...), the others as
// harness::<op>::run_<op>_cpu(...).  This header keeps those namespaces, names and argument
// meanings and adds, per operator:
//   * the same host-pointer fp32 call, executed on the GPU (`run` / `run_<op>_cuda`): device
//     buffers are allocated, inputs copied in, the CUDA kernel launched and the outputs copied
//     back before the call returns;
//   * a device-pointer call (`run_device` / `run_<op>_device`) for fp32, fp16 or bf16 buffers,
//     asynchronous on a CUDA stream (passed as void*, nullptr = default stream);
//   * for flash attention, a 16-bit host-buffer call that pipelines copies with the kernel.
//
// Error behaviour: a failure (no device, an argument the kernel cannot take, a CUDA error, an
// expired bounded wait) throws harness::DeviceError carrying the hc_status code and message.
// There is no CPU fallback: the reference runners fell back to the golden when no device was
// present (ops/elementwise_add/runner/elementwise_add_runner.cpp:40-41); these report instead,
// so a result always comes from the GPU.
#pragma once

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <utility>

#include "hc_ops.h"

namespace harness {

class DeviceError : public std::runtime_error {
public:
    DeviceError(int status, const std::string& what) : std::runtime_error(what), status_(status) {}
    int status() const { return status_; }

private:
    int status_;
};

namespace device {

// Element types, numbered like hc_dtype (and the reference's harness::Dtype).
enum class Dtype : int {
    F32 = HC_DTYPE_F32,
    F16 = HC_DTYPE_F16,
    BF16 = HC_DTYPE_BF16,
    I32 = HC_DTYPE_I32,
    I8 = HC_DTYPE_I8,
    U8 = HC_DTYPE_U8,
};

// Throws DeviceError(status, "<what>: <last error message>") unless status == HC_OK.
void ThrowIfError(int status, const char* what);

namespace detail {
// Element count of a shape object (anything with num_elements(), e.g. the reference's
// harness::Shape) or of a plain count.
inline size_t elems(size_t n) { return n; }
template <class S, class = decltype(std::declval<const S&>().num_elements())>
size_t elems(const S& s) {
    return static_cast<size_t>(s.num_elements());
}
template <class E>
int as_int(E e) {
    return static_cast<int>(e);
}
}  // namespace detail

}  // namespace device

// ================================================================ elementwise family
namespace runner {

namespace elementwise_add {
// z = x + y (ops/elementwise_add/runner/elementwise_add_runner.hpp:15).
void run(const float* x, const float* y, float* z, size_t n);
template <class S, class = decltype(std::declval<const S&>().num_elements())>
void run(const float* x, const float* y, float* z, const S& shape) {
    run(x, y, z, device::detail::elems(shape));
}
void run_device(const void* x, const void* y, void* z, size_t n, device::Dtype dtype, void* stream = nullptr);
}  // namespace elementwise_add

namespace axpy_scalar_affine {
// y = alpha * x + beta (ops/axpy_scalar_affine/runner/axpy_scalar_affine_runner.hpp:11).
void run(const float* x, float* y, size_t n, float alpha, float beta);
template <class S, class = decltype(std::declval<const S&>().num_elements())>
void run(const float* x, float* y, const S& shape, float alpha, float beta) {
    run(x, y, device::detail::elems(shape), alpha, beta);
}
void run_device(const void* x, void* y, size_t n, float alpha, float beta, device::Dtype dtype,
                void* stream = nullptr);
}  // namespace axpy_scalar_affine

namespace broadcast_binary {
// z[b,c,h,w] = x[b,c,h,w] * y[yb,c] + bias[c], NCHW, y_batch 1 or B
// (ops/broadcast_binary/runner/broadcast_binary_runner.hpp:14-15).
void run(const float* x, const float* y, const float* bias, float* z, int64_t B, int64_t C, int64_t H,
         int64_t W, int64_t y_batch);
void run_device(const void* x, const void* y, const void* bias, void* z, int64_t B, int64_t C, int64_t H,
                int64_t W, int64_t y_batch, device::Dtype dtype, void* stream = nullptr);
}  // namespace broadcast_binary

namespace activation_gelu_silu {
// y = GELU_tanh(x) (act 0) or SiLU(x) (act 1)
// (ops/activation_gelu_silu/runner/activation_gelu_silu_runner.hpp:10).  `act` may be the
// reference's golden::activation_gelu_silu::ActivationType or an int.
void run(const float* x, float* y, size_t n, int act);
template <class SizeOrShape, class Act>
void run(const float* x, float* y, const SizeOrShape& shape, Act act) {
    run(x, y, device::detail::elems(shape), device::detail::as_int(act));
}
void run_device(const void* x, void* y, size_t n, int act, device::Dtype dtype, void* stream = nullptr);
}  // namespace activation_gelu_silu

namespace reduce_sum_lastdim {
// out[b,m] = sum_k x[b,m,k] (ops/reduce_sum_lastdim/runner/reduce_sum_lastdim_runner.hpp:15-16).
void run(const float* x, float* out, int64_t num_batches, int64_t M, int64_t K);
// x of `dtype`, out always fp32.
void run_device(const void* x, float* out, int64_t num_batches, int64_t M, int64_t K, device::Dtype dtype,
                void* stream = nullptr);
}  // namespace reduce_sum_lastdim

}  // namespace runner

// ================================================================ transpose
namespace transpose_2d_4d {
// Index permutations, bit-exact for any element type of 1, 2 or 4 bytes
// (ops/transpose_2d_4d/runner/transpose_2d_4d_runner.hpp:10-26).
// mode 0: [M,N] -> [N,M] (d0 = M, d1 = N); mode 1: NCHW -> NHWC; mode 2: NHWC -> NCHW
// (d0..d3 = N, C, H, W).
void run_transpose_device(const void* src, void* dst, int mode, int64_t d0, int64_t d1, int64_t d2, int64_t d3,
                          size_t elem_bytes, void* stream = nullptr);
void run_transpose_host(const void* src, void* dst, int mode, int64_t d0, int64_t d1, int64_t d2, int64_t d3,
                        size_t elem_bytes);

template <typename T>
void run_transpose_2d_cuda(const T* input, T* output, int64_t M, int64_t N) {
    static_assert(sizeof(T) == 1 || sizeof(T) == 2 || sizeof(T) == 4, "element size 1, 2 or 4 bytes");
    run_transpose_host(input, output, 0, M, N, 1, 1, sizeof(T));
}
template <typename T>
void run_transpose_4d_nchw_to_nhwc_cuda(const T* input, T* output, int64_t N, int64_t C, int64_t H, int64_t W) {
    static_assert(sizeof(T) == 1 || sizeof(T) == 2 || sizeof(T) == 4, "element size 1, 2 or 4 bytes");
    run_transpose_host(input, output, 1, N, C, H, W, sizeof(T));
}
template <typename T>
void run_transpose_4d_nhwc_to_nchw_cuda(const T* input, T* output, int64_t N, int64_t C, int64_t H, int64_t W) {
    static_assert(sizeof(T) == 1 || sizeof(T) == 2 || sizeof(T) == 4, "element size 1, 2 or 4 bytes");
    run_transpose_host(input, output, 2, N, C, H, W, sizeof(T));
}
}  // namespace transpose_2d_4d

// ================================================================ layer_norm
namespace layer_norm {
// y = (x - mean) / sqrt(var + eps) * gamma + beta over the last dim
// (ops/layer_norm/runner/layer_norm_runner.hpp:10-13).  gamma/beta fp32.
void run_layer_norm_cuda(const float* x, const float* gamma, const float* beta, float* y, int64_t rows,
                         int64_t last_dim, float eps);
void run_layer_norm_device(const void* x, const float* gamma, const float* beta, void* y, int64_t rows,
                           int64_t last_dim, float eps, device::Dtype dtype, void* stream = nullptr);
}  // namespace layer_norm

// ================================================================ rms_norm_rope_fused
namespace rms_norm_rope_fused {
enum class RopeStyle : uint32_t {
    Interleaved = 0,  // pairs (2d, 2d+1), as the reference golden
    RotateHalf = 1,   // pairs (d, d + rotary_dim/2)
};
// RMSNorm over H, then interleaved RoPE on the first rotary_dim elements, x/out [B, S, H]
// (ops/rms_norm_rope_fused/runner/rms_norm_rope_fused_runner.hpp:10-17).  cos/sin [S, rotary_dim/2].
void run_rms_norm_rope_fused_cuda(const float* x, const float* weight, const float* cos, const float* sin,
                                  float* out, int64_t B, int64_t S, int64_t H, int64_t rotary_dim, float eps);
// Same on device buffers; `heads` > 1 gives x/out [B, S, heads, H] (every head of a position
// shares its cos/sin row).
void run_rms_norm_rope_fused_device(const void* x, const float* weight, const float* cos, const float* sin,
                                    void* out, int64_t B, int64_t S, int64_t H, int64_t rotary_dim, float eps,
                                    int64_t heads, RopeStyle style, device::Dtype dtype, void* stream = nullptr);
}  // namespace rms_norm_rope_fused

// ================================================================ matmul_bias
namespace matmul_bias {
// C[M,N] = A[M,K] . B[K,N] + bias[N] (bias may be nullptr)
// (ops/matmul_bias/runner/matmul_bias_runner.hpp:10-15).  fp32 runs the SIMT kernel;
// bf16/fp16 device buffers run the tcgen05 kernel.
void run_matmul_bias_cuda(const float* A, const float* B, const float* bias, float* C, int64_t M, int64_t K,
                          int64_t N);
void run_matmul_bias_device(const void* A, const void* B, const void* bias, void* C, int64_t M, int64_t K,
                            int64_t N, device::Dtype dtype, void* stream = nullptr);
}  // namespace matmul_bias

// ================================================================ flash_attention_fwd_fused
namespace flash_attention_fwd_fused {
// O = softmax(Q K^T * scale [+ causal mask]) V, Q [B,H,S_q,D], K [B,H,S_k,D], V [B,H,S_k,D_v]
// (ops/flash_attention_fwd_fused/runner/flash_attention_fwd_fused_runner.hpp:9-18).
// mask_type 0 = none, 1 = causal (top-left aligned); the reference's AttnMaskType converts.
void run_flash_attention_fwd_fused_cuda(const float* Q, const float* K, const float* V, float* O, int64_t B,
                                        int64_t H, int64_t S_q, int64_t S_k, int64_t D, int64_t D_v, float scale,
                                        int mask_type);
template <class Mask, class = std::enable_if_t<!std::is_same<Mask, int>::value>>
void run_flash_attention_fwd_fused_cuda(const float* Q, const float* K, const float* V, float* O, int64_t B,
                                        int64_t H, int64_t S_q, int64_t S_k, int64_t D, int64_t D_v, float scale,
                                        Mask mask_type) {
    run_flash_attention_fwd_fused_cuda(Q, K, V, O, B, H, S_q, S_k, D, D_v, scale, device::detail::as_int(mask_type));
}
// Device buffers; lse [B,H,S_q] fp32 (natural log) may be nullptr.  bf16/fp16 with D and D_v
// each 64 or 128 runs the tcgen05/TMEM kernel.
void run_flash_attention_fwd_fused_device(const void* q, const void* k, const void* v, void* o, float* lse,
                                          int64_t B, int64_t H, int64_t S_q, int64_t S_k, int64_t D, int64_t D_v,
                                          float scale, int mask_type, device::Dtype dtype, void* stream = nullptr);
// Grouped-query form (no counterpart in the reference): K and V hold kv_heads heads, a divisor of
// H, and query head h reads K/V head h / (H / kv_heads).
void run_flash_attention_fwd_fused_gqa_device(const void* q, const void* k, const void* v, void* o, float* lse,
                                              int64_t B, int64_t H, int64_t kv_heads, int64_t S_q, int64_t S_k,
                                              int64_t D, int64_t D_v, float scale, int mask_type, device::Dtype dtype,
                                              void* stream = nullptr);
// Host buffers of `dtype` (pinned for full copy bandwidth); copies are pipelined with the kernel
// over chunks of heads.  Synchronous: returns when o and lse are in host memory.
void run_flash_attention_fwd_fused_host(const void* q, const void* k, const void* v, void* o, float* lse,
                                        int64_t B, int64_t H, int64_t S_q, int64_t S_k, int64_t D, int64_t D_v,
                                        float scale, int mask_type, device::Dtype dtype, void* stream = nullptr);
}  // namespace flash_attention_fwd_fused

}  // namespace harness
