// extern "C" wrappers around the reference harness's own golden functions -- TEST
// INFRASTRUCTURE ONLY.  Compiled by oracle/Makefile together with the unchanged golden sources
// from the reference tree into oracle/_ref/libref_golden.so; used to pin the oracle restatement
// (tests/golden/make_golden.py) and as the reference CPU arm of bench.py.
#include <cstring>
#include <thread>
#include <vector>

#include "activation_gelu_silu_golden.hpp"
#include "axpy_scalar_affine_golden.hpp"
#include "broadcast_binary_golden.hpp"
#include "elementwise_add_golden.hpp"
#include "flash_attention_fwd_fused_golden.hpp"
#include "harness/test_utils.hpp"
#include "layer_norm_golden.hpp"
#include "matmul_bias_golden.hpp"
#include "reduce_sum_lastdim_golden.hpp"
#include "rms_norm_rope_fused_golden.hpp"
#include "transpose_2d_4d_golden.hpp"

extern "C" {

void ref_generate_random_float(float* out, size_t n, uint64_t seed, float lo, float hi) {
    std::vector<float> v = harness::test::generate_random_float(n, seed, lo, hi);
    std::memcpy(out, v.data(), n * sizeof(float));
}

void ref_generate_rope_cos_sin(size_t seq_len, size_t half, float* cos_out, float* sin_out, float base) {
    std::vector<float> c, s;
    harness::test::generate_rope_cos_sin(seq_len, half, c, s, base);
    std::memcpy(cos_out, c.data(), c.size() * sizeof(float));
    std::memcpy(sin_out, s.data(), s.size() * sizeof(float));
}

void ref_elementwise_add(const float* x, const float* y, float* z, size_t n) {
    harness::golden::elementwise_add::compute(x, y, z, n);
}

void ref_axpy_scalar_affine(const float* x, float* y, size_t n, float alpha, float beta) {
    harness::golden::axpy_scalar_affine::compute(x, y, n, alpha, beta);
}

void ref_broadcast_binary(const float* x, const float* y, const float* bias, float* z, int64_t B, int64_t C, int64_t H,
                          int64_t W, int64_t y_batch) {
    harness::golden::broadcast_binary::compute(x, y, bias, z, B, C, H, W, y_batch);
}

void ref_activation_gelu_silu(const float* x, float* y, size_t n, int act) {
    harness::golden::activation_gelu_silu::compute(
        x, y, n, act == 0 ? harness::golden::activation_gelu_silu::ActivationType::GELU
                          : harness::golden::activation_gelu_silu::ActivationType::SiLU);
}

void ref_reduce_sum_lastdim(const float* x, float* out, int64_t batches, int64_t M, int64_t K) {
    harness::golden::reduce_sum_lastdim::compute(x, out, batches, M, K);
}

// mode 0: 2D [M,N]; mode 1: NCHW->NHWC; mode 2: NHWC->NCHW.  is_int selects the int32 instance.
void ref_transpose(const void* in, void* out, int mode, int64_t d0, int64_t d1, int64_t d2, int64_t d3, int is_int) {
    using namespace harness::transpose_2d_4d;
    if (is_int) {
        const int32_t* i = static_cast<const int32_t*>(in);
        int32_t* o = static_cast<int32_t*>(out);
        if (mode == 0) transpose_2d_golden<int32_t>(i, o, d0, d1);
        else if (mode == 1) transpose_4d_nchw_to_nhwc_golden<int32_t>(i, o, d0, d1, d2, d3);
        else transpose_4d_nhwc_to_nchw_golden<int32_t>(i, o, d0, d1, d2, d3);
    } else {
        const float* i = static_cast<const float*>(in);
        float* o = static_cast<float*>(out);
        if (mode == 0) transpose_2d_golden<float>(i, o, d0, d1);
        else if (mode == 1) transpose_4d_nchw_to_nhwc_golden<float>(i, o, d0, d1, d2, d3);
        else transpose_4d_nhwc_to_nchw_golden<float>(i, o, d0, d1, d2, d3);
    }
}

void ref_layer_norm(const float* x, const float* gamma, const float* beta, float* y, int64_t rows, int64_t last_dim,
                    float eps) {
    harness::layer_norm::layer_norm_golden(x, gamma, beta, y, rows, last_dim, eps);
}

void ref_rms_norm_rope_fused(const float* x, const float* w, const float* cos_t, const float* sin_t, float* out,
                             int64_t B, int64_t S, int64_t H, int64_t rot, float eps) {
    harness::rms_norm_rope_fused::rms_norm_rope_fused_golden(x, w, cos_t, sin_t, out, B, S, H, rot, eps);
}

void ref_matmul_bias(const float* A, const float* B, const float* bias, float* C, int64_t M, int64_t K, int64_t N) {
    harness::matmul_bias::matmul_bias_golden(A, B, bias, C, M, K, N);
}

void ref_flash_attention_fwd(const float* Q, const float* K, const float* V, float* O, int64_t B, int64_t H,
                             int64_t S_q, int64_t S_k, int64_t D, int64_t D_v, float scale, int mask) {
    harness::flash_attention_fwd_fused::flash_attention_fwd_golden(
        Q, K, V, O, B, H, S_q, S_k, D, D_v, scale,
        mask ? harness::flash_attention_fwd_fused::AttnMaskType::Causal
             : harness::flash_attention_fwd_fused::AttnMaskType::None);
}

// The golden over (b,h) heads split across `threads` host threads (each call sees B=1, H=range).
void ref_flash_attention_fwd_mt(const float* Q, const float* K, const float* V, float* O, int64_t B, int64_t H,
                                int64_t S_q, int64_t S_k, int64_t D, int64_t D_v, float scale, int mask, int threads) {
    const int64_t BH = B * H;
    if (threads < 1) threads = 1;
    if (threads > BH) threads = static_cast<int>(BH);
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; ++t) {
        int64_t h0 = BH * t / threads, h1 = BH * (t + 1) / threads;
        if (h1 <= h0) continue;
        pool.emplace_back([=] {
            ref_flash_attention_fwd(Q + h0 * S_q * D, K + h0 * S_k * D, V + h0 * S_k * D_v, O + h0 * S_q * D_v, 1,
                                    h1 - h0, S_q, S_k, D, D_v, scale, mask);
        });
    }
    for (auto& th : pool) th.join();
}

}  // extern "C"
