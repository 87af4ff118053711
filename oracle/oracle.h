/*
 * oracle.h -- CPU restatement of the reference harness's golden functions.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links, loads or calls this code.
 * The CUDA kernels are compared against it (tests/), bench.py times it as the CPU baseline, and
 * __graft_entry__.smoke() checks its one launch with it.  Each function cites the golden it restates
 * (paths are inside the z-zijie/ascend-npu-harness project).  Parity with the reference itself
 * is pinned by tests/test_oracle_pins.py against fixtures produced by the reference's own
 * golden sources (oracle/Makefile builds them into oracle/_ref/).
 */
#ifndef HC_ORACLE_H
#define HC_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- data generation (include/harness/test_utils.hpp) ---- */
/* mt19937_64(seed) + uniform_real_distribution<float>(lo, hi): test_utils.hpp:39-46 */
void oracle_uniform_f32(float* out, size_t n, uint64_t seed, float lo, float hi);
/* N(mean, std) by the Box-Muller transform on mt19937_64 doubles (no reference counterpart;
 * the harness has no normal generator, test_utils.hpp:18-142). */
void oracle_normal_f32(float* out, size_t n, uint64_t seed, float mean, float stddev);
/* RoPE tables cos/sin[s, d] for theta = s / base^(2d / (2*half)): test_utils.hpp:59-72 */
void oracle_rope_cos_sin(size_t seq_len, size_t half, float* cos_out, float* sin_out, float base);

/* ---- 16-bit float codecs (IEEE-754 round-to-nearest-even, subnormals kept) ---- */
void oracle_f32_to_bf16(const float* in, uint16_t* out, size_t n);
void oracle_bf16_to_f32(const uint16_t* in, float* out, size_t n);
void oracle_f32_to_f16(const float* in, uint16_t* out, size_t n);
void oracle_f16_to_f32(const uint16_t* in, float* out, size_t n);

/* ---- the ten ladder goldens ---- */
/* ops/elementwise_add/golden/elementwise_add_golden.cpp:8-15 */
void oracle_elementwise_add(const float* x, const float* y, float* z, size_t n);
/* ops/axpy_scalar_affine/golden/axpy_scalar_affine_golden.cpp:8-16 */
void oracle_axpy_scalar_affine(const float* x, float* y, size_t n, float alpha, float beta);
/* ops/broadcast_binary/golden/broadcast_binary_golden.cpp:8-41 */
void oracle_broadcast_binary(const float* x, const float* y, const float* bias, float* z, int64_t B, int64_t C,
                             int64_t H, int64_t W, int64_t y_batch);
/* ops/activation_gelu_silu/golden/activation_gelu_silu_golden.cpp:16-49; act 0 GELU, 1 SiLU */
void oracle_activation_gelu_silu(const float* x, float* y, size_t n, int act);
/* ops/reduce_sum_lastdim/golden/reduce_sum_lastdim_golden.cpp:10-46 */
void oracle_reduce_sum_lastdim(const float* x, float* out, int64_t batches, int64_t M, int64_t K);
/* ops/transpose_2d_4d/golden/transpose_2d_4d_golden.cpp:7-62; elem_bytes 1, 2, 4 or 8.
 * mode 0: [M,N] -> [N,M]; mode 1: NCHW -> NHWC; mode 2: NHWC -> NCHW (d0..d3 = N,C,H,W). */
void oracle_transpose(const void* in, void* out, int mode, int64_t d0, int64_t d1, int64_t d2, int64_t d3,
                      int elem_bytes);
/* ops/layer_norm/golden/layer_norm_golden.cpp:8-41 */
void oracle_layer_norm(const float* x, const float* gamma, const float* beta, float* y, int64_t rows,
                       int64_t last_dim, float eps);
/* ops/rms_norm_rope_fused/golden/rms_norm_rope_fused_golden.cpp:8-55, generalised to rows of
 * `heads` heads per sequence position (position = (row / heads) % S) and to the rotate-half
 * pairing (style 1: (d, d + rot/2)); style 0 with heads 1 is the golden itself. */
void oracle_rms_norm_rope(const float* x, const float* weight, const float* cos_t, const float* sin_t, float* out,
                          int64_t rows, int64_t H, int64_t rot, float eps, int64_t heads, int64_t S, int style);
/* ops/matmul_bias/golden/matmul_bias_golden.cpp:6-27 (bias may be NULL) */
void oracle_matmul_bias(const float* A, const float* B, const float* bias, float* C, int64_t M, int64_t K,
                        int64_t N);
/* Flash-attention backward in fp64: exact dQ, dK, dV of softmax(Q K^T * scale [causal]) V for dO (the
 * harness has no backward golden; this restates the gradients from the definition). */
void oracle_flash_attention_bwd(const float* Q, const float* K, const float* V, const float* dO, float* dQ, float* dK,
                                float* dV, int64_t B, int64_t H, int64_t S_q, int64_t S_k, int64_t D, int64_t D_v,
                                float scale, int mask);
/* ops/flash_attention_fwd_fused/golden/flash_attention_fwd_fused_golden.cpp:10-112, plus
 * lse = m + ln(l) per row (may be NULL).  mask 0 none, 1 causal. */
void oracle_flash_attention_fwd(const float* Q, const float* K, const float* V, float* O, float* lse, int64_t B,
                                int64_t H, int64_t S_q, int64_t S_k, int64_t D, int64_t D_v, float scale, int mask);
/* Same, heads split over `threads` host threads (bench CPU baseline). */
void oracle_flash_attention_fwd_mt(const float* Q, const float* K, const float* V, float* O, float* lse, int64_t B,
                                   int64_t H, int64_t S_q, int64_t S_k, int64_t D, int64_t D_v, float scale, int mask,
                                   int threads);

#ifdef __cplusplus
}
#endif

#endif
