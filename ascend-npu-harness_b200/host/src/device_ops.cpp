// harness runners on top of the C-ABI (hc_ops.h / hc_runtime.h).  Host-pointer calls allocate
// device buffers, copy in, launch on the default stream, copy out and check the device error
// words; device-pointer calls only fill the tiling record and launch.  Every failure throws
// harness::DeviceError; nothing here computes on the CPU.
#include "harness/device_ops.hpp"

#include <cstring>
#include <limits>
#include <string>

#include "hc_runtime.h"

namespace harness {
namespace device {

void ThrowIfError(int status, const char* what) {
    if (status == HC_OK) return;
    const char* msg = hc_last_error_string();
    throw DeviceError(status, std::string(what) + ": " + (msg && *msg ? msg : "error " + std::to_string(status)));
}

}  // namespace device

namespace {

using device::Dtype;
using device::ThrowIfError;

uint32_t u32(int64_t v, const char* what) {
    if (v < 0 || v > static_cast<int64_t>(std::numeric_limits<uint32_t>::max()))
        throw DeviceError(HC_ERR_INVALID, std::string(what) + ": extent " + std::to_string(v) +
                                              " outside [0, 2^32) (tiling fields are 32-bit)");
    return static_cast<uint32_t>(v);
}

uint32_t u32(size_t v, const char* what) {
    if (v > std::numeric_limits<uint32_t>::max())
        throw DeviceError(HC_ERR_INVALID, std::string(what) + ": " + std::to_string(v) +
                                              " elements do not fit the 32-bit tiling field");
    return static_cast<uint32_t>(v);
}

void require_device(const char* what) {
    int n = 0;
    if (hc_device_count(&n) != HC_OK || n == 0)
        throw DeviceError(HC_ERR_NO_DEVICE, std::string(what) + ": no CUDA device (there is no CPU fallback)");
}

// A device buffer owned for the duration of one host-pointer call.
class Scratch {
public:
    Scratch(size_t bytes, const char* what) : bytes_(bytes) {
        if (bytes) ThrowIfError(hc_malloc(&p_, bytes), what);
    }
    ~Scratch() {
        if (p_) hc_free(p_);
    }
    Scratch(Scratch&& o) noexcept : p_(o.p_), bytes_(o.bytes_) {
        o.p_ = nullptr;
        o.bytes_ = 0;
    }
    Scratch(const Scratch&) = delete;
    Scratch& operator=(const Scratch&) = delete;
    Scratch& operator=(Scratch&&) = delete;
    void* get() const { return p_; }
    template <class T>
    T* as() const {
        return static_cast<T*>(p_);
    }
    void upload(const void* host, const char* what) {
        if (bytes_ && host) ThrowIfError(hc_memcpy_h2d(p_, host, bytes_, nullptr), what);
    }
    void download(void* host, const char* what) const {
        if (bytes_) ThrowIfError(hc_memcpy_d2h(host, p_, bytes_, nullptr), what);
    }

private:
    void* p_ = nullptr;
    size_t bytes_;
};

Scratch upload(const void* host, size_t bytes, const char* what) {
    Scratch s(bytes, what);
    s.upload(host, what);
    return s;
}

// Waits for the launch and reports a CUDA error or an expired bounded wait.
void finish(const char* what) {
    ThrowIfError(hc_device_sync(), what);
    ThrowIfError(hc_check_device_error(), what);
}

}  // namespace

// ================================================================ elementwise_add
namespace runner {
namespace elementwise_add {

void run_device(const void* x, const void* y, void* z, size_t n, Dtype dtype, void* stream) {
    const char* what = "elementwise_add";
    elementwise_add_tiling_data t{u32(n, what), 0};
    if (n == 0) return;
    ThrowIfError(hc_elementwise_add_launch(x, y, z, &t, static_cast<int>(dtype), stream), what);
}

void run(const float* x, const float* y, float* z, size_t n) {
    const char* what = "elementwise_add";
    u32(n, what);
    require_device(what);
    if (n == 0) return;
    const size_t bytes = n * sizeof(float);
    Scratch dx = upload(x, bytes, what), dy = upload(y, bytes, what), dz(bytes, what);
    run_device(dx.get(), dy.get(), dz.get(), n, Dtype::F32, nullptr);
    dz.download(z, what);
    finish(what);
}

}  // namespace elementwise_add

// ================================================================ axpy_scalar_affine
namespace axpy_scalar_affine {

void run_device(const void* x, void* y, size_t n, float alpha, float beta, Dtype dtype, void* stream) {
    const char* what = "axpy_scalar_affine";
    axpy_scalar_affine_tiling_data t{u32(n, what), 0};
    if (n == 0) return;
    ThrowIfError(hc_axpy_scalar_affine_launch(x, y, &t, alpha, beta, static_cast<int>(dtype), stream), what);
}

void run(const float* x, float* y, size_t n, float alpha, float beta) {
    const char* what = "axpy_scalar_affine";
    u32(n, what);
    require_device(what);
    if (n == 0) return;
    const size_t bytes = n * sizeof(float);
    Scratch dx = upload(x, bytes, what), dy(bytes, what);
    run_device(dx.get(), dy.get(), n, alpha, beta, Dtype::F32, nullptr);
    dy.download(y, what);
    finish(what);
}

}  // namespace axpy_scalar_affine

// ================================================================ broadcast_binary
namespace broadcast_binary {

void run_device(const void* x, const void* y, const void* bias, void* z, int64_t B, int64_t C, int64_t H, int64_t W,
                int64_t y_batch, Dtype dtype, void* stream) {
    const char* what = "broadcast_binary";
    broadcast_binary_tiling_data t{u32(B, what), u32(C, what), u32(H, what), u32(W, what), u32(y_batch, what), 0};
    if (B * C * H * W == 0) return;
    ThrowIfError(hc_broadcast_binary_launch(x, y, bias, z, &t, static_cast<int>(dtype), stream), what);
}

void run(const float* x, const float* y, const float* bias, float* z, int64_t B, int64_t C, int64_t H, int64_t W,
         int64_t y_batch) {
    const char* what = "broadcast_binary";
    const size_t n = static_cast<size_t>(u32(B, what)) * u32(C, what) * u32(H, what) * u32(W, what);
    u32(n, what);
    if (y_batch != 1 && y_batch != B)
        throw DeviceError(HC_ERR_INVALID, "broadcast_binary: y_batch must be 1 or B");
    require_device(what);
    if (n == 0) return;
    Scratch dx = upload(x, n * 4, what), dy = upload(y, static_cast<size_t>(y_batch * C) * 4, what),
            db = upload(bias, static_cast<size_t>(C) * 4, what), dz(n * 4, what);
    run_device(dx.get(), dy.get(), db.get(), dz.get(), B, C, H, W, y_batch, Dtype::F32, nullptr);
    dz.download(z, what);
    finish(what);
}

}  // namespace broadcast_binary

// ================================================================ activation_gelu_silu
namespace activation_gelu_silu {

void run_device(const void* x, void* y, size_t n, int act, Dtype dtype, void* stream) {
    const char* what = "activation_gelu_silu";
    if (act != 0 && act != 1) throw DeviceError(HC_ERR_INVALID, "activation_gelu_silu: act must be 0 (GELU) or 1 (SiLU)");
    activation_gelu_silu_tiling_data t{u32(n, what), 0, static_cast<uint32_t>(act)};
    if (n == 0) return;
    ThrowIfError(hc_activation_gelu_silu_launch(x, y, &t, static_cast<int>(dtype), stream), what);
}

void run(const float* x, float* y, size_t n, int act) {
    const char* what = "activation_gelu_silu";
    u32(n, what);
    if (act != 0 && act != 1) throw DeviceError(HC_ERR_INVALID, "activation_gelu_silu: act must be 0 (GELU) or 1 (SiLU)");
    require_device(what);
    if (n == 0) return;
    const size_t bytes = n * sizeof(float);
    Scratch dx = upload(x, bytes, what), dy(bytes, what);
    run_device(dx.get(), dy.get(), n, act, Dtype::F32, nullptr);
    dy.download(y, what);
    finish(what);
}

}  // namespace activation_gelu_silu

// ================================================================ reduce_sum_lastdim
namespace reduce_sum_lastdim {

void run_device(const void* x, float* out, int64_t num_batches, int64_t M, int64_t K, Dtype dtype, void* stream) {
    const char* what = "reduce_sum_lastdim";
    reduce_sum_lastdim_tiling_data t{u32(num_batches * M, what), u32(K, what), 0};
    if (num_batches * M == 0) return;
    ThrowIfError(hc_reduce_sum_lastdim_launch(x, out, &t, static_cast<int>(dtype), stream), what);
}

void run(const float* x, float* out, int64_t num_batches, int64_t M, int64_t K) {
    const char* what = "reduce_sum_lastdim";
    const size_t rows = u32(num_batches * M, what);
    u32(K, what);
    require_device(what);
    if (rows == 0) return;
    Scratch dx = upload(x, rows * static_cast<size_t>(K) * 4, what), dout(rows * 4, what);
    run_device(dx.get(), dout.as<float>(), num_batches, M, K, Dtype::F32, nullptr);
    dout.download(out, what);
    finish(what);
}

}  // namespace reduce_sum_lastdim
}  // namespace runner

// ================================================================ transpose_2d_4d
namespace transpose_2d_4d {

namespace {
Dtype dtype_for_size(size_t elem_bytes) {
    switch (elem_bytes) {
        case 1: return Dtype::U8;
        case 2: return Dtype::F16;
        case 4: return Dtype::F32;
        default: throw DeviceError(HC_ERR_UNSUPPORTED, "transpose_2d_4d: element size must be 1, 2 or 4 bytes");
    }
}
}  // namespace

void run_transpose_device(const void* src, void* dst, int mode, int64_t d0, int64_t d1, int64_t d2, int64_t d3,
                          size_t elem_bytes, void* stream) {
    const char* what = "transpose_2d_4d";
    if (mode < 0 || mode > 2) throw DeviceError(HC_ERR_INVALID, "transpose_2d_4d: mode must be 0, 1 or 2");
    transpose_2d_4d_tiling_data t{static_cast<uint32_t>(mode), u32(d0, what), u32(d1, what),
                                  u32(mode == 0 ? 1 : d2, what), u32(mode == 0 ? 1 : d3, what), 0};
    const Dtype dt = dtype_for_size(elem_bytes);
    if (d0 * d1 * (mode == 0 ? 1 : d2 * d3) == 0) return;
    ThrowIfError(hc_transpose_2d_4d_launch(src, dst, &t, static_cast<int>(dt), stream), what);
}

void run_transpose_host(const void* src, void* dst, int mode, int64_t d0, int64_t d1, int64_t d2, int64_t d3,
                        size_t elem_bytes) {
    const char* what = "transpose_2d_4d";
    dtype_for_size(elem_bytes);
    const int64_t n = d0 * d1 * (mode == 0 ? 1 : d2 * d3);
    u32(n, what);
    require_device(what);
    if (n == 0) return;
    const size_t bytes = static_cast<size_t>(n) * elem_bytes;
    Scratch ds = upload(src, bytes, what), dd(bytes, what);
    run_transpose_device(ds.get(), dd.get(), mode, d0, d1, d2, d3, elem_bytes, nullptr);
    dd.download(dst, what);
    finish(what);
}

}  // namespace transpose_2d_4d

// ================================================================ layer_norm
namespace layer_norm {

void run_layer_norm_device(const void* x, const float* gamma, const float* beta, void* y, int64_t rows,
                           int64_t last_dim, float eps, Dtype dtype, void* stream) {
    const char* what = "layer_norm";
    layer_norm_tiling_data t{u32(rows, what), u32(last_dim, what), 0, eps};
    if (rows == 0) return;
    ThrowIfError(hc_layer_norm_launch(x, gamma, beta, y, &t, static_cast<int>(dtype), stream), what);
}

void run_layer_norm_cuda(const float* x, const float* gamma, const float* beta, float* y, int64_t rows,
                         int64_t last_dim, float eps) {
    const char* what = "layer_norm";
    u32(rows * last_dim, what);
    require_device(what);
    if (rows == 0) return;
    const size_t n = static_cast<size_t>(rows * last_dim);
    Scratch dx = upload(x, n * 4, what), dg = upload(gamma, static_cast<size_t>(last_dim) * 4, what),
            db = upload(beta, static_cast<size_t>(last_dim) * 4, what), dy(n * 4, what);
    run_layer_norm_device(dx.get(), dg.as<float>(), db.as<float>(), dy.get(), rows, last_dim, eps, Dtype::F32,
                          nullptr);
    dy.download(y, what);
    finish(what);
}

}  // namespace layer_norm

// ================================================================ rms_norm_rope_fused
namespace rms_norm_rope_fused {

void run_rms_norm_rope_fused_device(const void* x, const float* weight, const float* cos, const float* sin, void* out,
                                    int64_t B, int64_t S, int64_t H, int64_t rotary_dim, float eps, int64_t heads,
                                    RopeStyle style, Dtype dtype, void* stream) {
    const char* what = "rms_norm_rope_fused";
    rms_norm_rope_fused_tiling_data t{u32(B, what), u32(S, what), u32(H, what), u32(rotary_dim, what), 0, eps};
    if (B * S * H * heads == 0) return;
    ThrowIfError(hc_rms_norm_rope_fused_launch(x, weight, cos, sin, out, &t, u32(heads, what),
                                               static_cast<uint32_t>(style), static_cast<int>(dtype), stream),
                 what);
}

void run_rms_norm_rope_fused_cuda(const float* x, const float* weight, const float* cos, const float* sin,
                                  float* out, int64_t B, int64_t S, int64_t H, int64_t rotary_dim, float eps) {
    const char* what = "rms_norm_rope_fused";
    u32(B * S * H, what);
    if (rotary_dim < 0 || rotary_dim > H || rotary_dim % 2)
        throw DeviceError(HC_ERR_INVALID, "rms_norm_rope_fused: rotary_dim must be even and <= H");
    require_device(what);
    if (B * S * H == 0) return;
    const size_t n = static_cast<size_t>(B * S * H);
    const size_t table = static_cast<size_t>(S * (rotary_dim / 2)) * 4;
    Scratch dx = upload(x, n * 4, what), dw = upload(weight, static_cast<size_t>(H) * 4, what),
            dc = upload(cos, table, what), ds = upload(sin, table, what), dy(n * 4, what);
    run_rms_norm_rope_fused_device(dx.get(), dw.as<float>(), dc.as<float>(), ds.as<float>(), dy.get(), B, S, H,
                                   rotary_dim, eps, 1, RopeStyle::Interleaved, Dtype::F32, nullptr);
    dy.download(out, what);
    finish(what);
}

}  // namespace rms_norm_rope_fused

// ================================================================ matmul_bias
namespace matmul_bias {

void run_matmul_bias_device(const void* A, const void* B, const void* bias, void* C, int64_t M, int64_t K, int64_t N,
                            Dtype dtype, void* stream) {
    const char* what = "matmul_bias";
    matmul_bias_tiling_data t{u32(M, what), u32(K, what), u32(N, what), 0, 0, 0};
    if (M * N == 0) return;
    ThrowIfError(hc_matmul_bias_launch(A, B, bias, C, &t, static_cast<int>(dtype), stream), what);
}

void run_matmul_bias_cuda(const float* A, const float* B, const float* bias, float* C, int64_t M, int64_t K,
                          int64_t N) {
    const char* what = "matmul_bias";
    u32(M * K, what);
    u32(K * N, what);
    u32(M * N, what);
    require_device(what);
    if (M * N == 0) return;
    Scratch dA = upload(A, static_cast<size_t>(M * K) * 4, what), dB = upload(B, static_cast<size_t>(K * N) * 4, what),
            dbias(bias ? static_cast<size_t>(N) * 4 : 0, what), dC(static_cast<size_t>(M * N) * 4, what);
    if (bias) dbias.upload(bias, what);
    run_matmul_bias_device(dA.get(), dB.get(), bias ? dbias.get() : nullptr, dC.get(), M, K, N, Dtype::F32, nullptr);
    dC.download(C, what);
    finish(what);
}

}  // namespace matmul_bias

// ================================================================ flash_attention_fwd_fused
namespace flash_attention_fwd_fused {

namespace {
flash_attention_fwd_fused_tiling_data fa_tiling(int64_t B, int64_t H, int64_t S_q, int64_t S_k, int64_t D, int64_t D_v,
                                                float scale, int mask_type) {
    const char* what = "flash_attention_fwd_fused";
    if (mask_type != 0 && mask_type != 1)
        throw DeviceError(HC_ERR_INVALID, "flash_attention_fwd_fused: mask_type must be 0 (none) or 1 (causal)");
    return flash_attention_fwd_fused_tiling_data{u32(B, what),   u32(H, what), u32(S_q, what),
                                                 u32(S_k, what), u32(D, what), u32(D_v, what),
                                                 scale,          static_cast<uint32_t>(mask_type)};
}
}  // namespace

void run_flash_attention_fwd_fused_device(const void* q, const void* k, const void* v, void* o, float* lse, int64_t B,
                                          int64_t H, int64_t S_q, int64_t S_k, int64_t D, int64_t D_v, float scale,
                                          int mask_type, Dtype dtype, void* stream) {
    const auto t = fa_tiling(B, H, S_q, S_k, D, D_v, scale, mask_type);
    if (B * H * S_q == 0) return;
    ThrowIfError(hc_flash_attention_fwd_fused_launch(q, k, v, o, lse, &t, static_cast<int>(dtype), stream),
                 "flash_attention_fwd_fused");
}

void run_flash_attention_fwd_fused_gqa_device(const void* q, const void* k, const void* v, void* o, float* lse, int64_t B,
                                              int64_t H, int64_t kv_heads, int64_t S_q, int64_t S_k, int64_t D,
                                              int64_t D_v, float scale, int mask_type, Dtype dtype, void* stream) {
    const char* what = "flash_attention_fwd_fused (grouped-query)";
    const auto t = fa_tiling(B, H, S_q, S_k, D, D_v, scale, mask_type);
    if (kv_heads <= 0 || H % kv_heads != 0)
        throw DeviceError(HC_ERR_INVALID, "flash_attention_fwd_fused: kv_heads must divide H");
    if (B * H * S_q == 0) return;
    ThrowIfError(hc_flash_attention_fwd_fused_gqa_launch(q, k, v, o, lse, &t, u32(kv_heads, what), static_cast<int>(dtype),
                                                         stream),
                 what);
}

void run_flash_attention_fwd_fused_cuda(const float* Q, const float* K, const float* V, float* O, int64_t B, int64_t H,
                                        int64_t S_q, int64_t S_k, int64_t D, int64_t D_v, float scale, int mask_type) {
    const char* what = "flash_attention_fwd_fused";
    fa_tiling(B, H, S_q, S_k, D, D_v, scale, mask_type);
    require_device(what);
    if (B * H * S_q == 0) return;
    const size_t bh = static_cast<size_t>(B * H);
    Scratch dq = upload(Q, bh * S_q * D * 4, what), dk = upload(K, bh * S_k * D * 4, what),
            dv = upload(V, bh * S_k * D_v * 4, what), dout(bh * S_q * D_v * 4, what);
    run_flash_attention_fwd_fused_device(dq.get(), dk.get(), dv.get(), dout.get(), nullptr, B, H, S_q, S_k, D, D_v,
                                         scale, mask_type, Dtype::F32, nullptr);
    dout.download(O, what);
    finish(what);
}

void run_flash_attention_fwd_fused_host(const void* q, const void* k, const void* v, void* o, float* lse, int64_t B,
                                        int64_t H, int64_t S_q, int64_t S_k, int64_t D, int64_t D_v, float scale,
                                        int mask_type, Dtype dtype, void* stream) {
    const char* what = "flash_attention_fwd_fused (host buffers)";
    const auto t = fa_tiling(B, H, S_q, S_k, D, D_v, scale, mask_type);
    require_device(what);
    if (B * H * S_q == 0) return;
    size_t ws = 0;
    ThrowIfError(hc_flash_attention_fwd_fused_host_workspace_size(&t, static_cast<int>(dtype), &ws), what);
    Scratch work(ws, what);
    ThrowIfError(hc_flash_attention_fwd_fused_host(q, k, v, o, lse, &t, static_cast<int>(dtype), work.get(), ws, stream),
                 what);
}

}  // namespace flash_attention_fwd_fused

}  // namespace harness
