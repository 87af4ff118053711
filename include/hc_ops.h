/*
 * hc_ops.h -- C-ABI kernel launches for the ten ladder operators on B200 (sm_100a).
 *
 * Each entry point replaces one AscendC kernel entry
 *   extern "C" __global__ __aicore__ <op>_kernel(GM_ADDR in..., GM_ADDR out..., GM_ADDR workspace,
 *                                                GM_ADDR tiling)
 * (docs/direct_launch.md:9-37 of the reference).  Differences, all deliberate:
 *   - the tiling POD is passed by host pointer and read on the host (it becomes kernel
 *     parameters); field layout and names are the reference's own host/<op>_tiling.h structs;
 *   - buffers carry an element type (hc_dtype) instead of being fp32-only;
 *   - the reference's AscendC "tileNum" field is accepted and ignored: the grid is sized
 *     from the SM count;
 *   - launches are asynchronous on `stream` (cudaStream_t as void*, NULL = default stream);
 *   - there is no workspace argument: no kernel here needs global scratch memory.
 *
 * Every launch validates its arguments on the host and returns HC_ERR_INVALID /
 * HC_ERR_UNSUPPORTED instead of running; there is no CPU fallback anywhere.
 * Status codes and hc_last_error_string() are declared in hc_runtime.h.
 */
#ifndef HC_OPS_H
#define HC_OPS_H

#include <stddef.h>
#include <stdint.h>

#include "hc_runtime.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------------------------
 * Tiling PODs.  Same fields, order and types as the reference's host/<op>_tiling.h.
 * ---------------------------------------------------------------------------------------- */

/* ops/elementwise_add/host/elementwise_add_tiling.h:4-7 */
struct elementwise_add_tiling_data {
    uint32_t totalLength;
    uint32_t tileNum;
};

/* ops/axpy_scalar_affine/host/axpy_scalar_affine_tiling.h:4-7 (alpha/beta are passed as
 * arguments: the reference kernel reads tilingData.alpha/.beta that its POD lacks,
 * ops/axpy_scalar_affine/kernel/axpy_scalar_affine_kernel.cpp:70). */
struct axpy_scalar_affine_tiling_data {
    uint32_t totalLength;
    uint32_t tileNum;
};

/* ops/broadcast_binary/host/broadcast_binary_tiling.h:5-12 */
struct broadcast_binary_tiling_data {
    uint32_t B;
    uint32_t C;
    uint32_t H;
    uint32_t W;
    uint32_t y_batch;  /* 1 (y broadcast over batch) or B */
    uint32_t tileNum;
};

/* ops/activation_gelu_silu/host/activation_gelu_silu_tiling.h:5-9 */
struct activation_gelu_silu_tiling_data {
    uint32_t totalLength;
    uint32_t tileNum;
    uint32_t actType;  /* 0 = GELU (tanh form), 1 = SiLU */
};

/* ops/reduce_sum_lastdim/host/reduce_sum_lastdim_tiling.h:5-9 */
struct reduce_sum_lastdim_tiling_data {
    uint32_t totalRows;  /* num_batches * M */
    uint32_t K;
    uint32_t tileNum;
};

/* ops/transpose_2d_4d/host/transpose_2d_4d_tiling.h:5-12 */
struct transpose_2d_4d_tiling_data {
    uint32_t mode;   /* 0 = 2D [M,N]->[N,M], 1 = NCHW->NHWC, 2 = NHWC->NCHW */
    uint32_t M;      /* 2D: M, 4D: N */
    uint32_t N_dim;  /* 2D: N, 4D: C */
    uint32_t H;      /* 4D only */
    uint32_t W;      /* 4D only */
    uint32_t tileNum;
};

/* ops/layer_norm/host/layer_norm_tiling.h:5-10 */
struct layer_norm_tiling_data {
    uint32_t rows;
    uint32_t lastDim;
    uint32_t tileNum;
    float eps;
};

/* ops/rms_norm_rope_fused/host/rms_norm_rope_fused_tiling.h:5-12.
 * H is the normalised (per-head) width; rows are B*S*(heads) of H elements each. */
struct rms_norm_rope_fused_tiling_data {
    uint32_t B;
    uint32_t S;
    uint32_t H;
    uint32_t rotaryDim;
    uint32_t tileNum;
    float eps;
};

/* ops/matmul_bias/host/matmul_bias_tiling.h:5-12 */
struct matmul_bias_tiling_data {
    uint32_t M;
    uint32_t K;
    uint32_t N;
    uint32_t tileM;
    uint32_t tileK;
    uint32_t tileN;
};

/* ops/flash_attention_fwd_fused/host/flash_attention_fwd_fused_tiling.h:5-14 */
struct flash_attention_fwd_fused_tiling_data {
    uint32_t B;
    uint32_t H;
    uint32_t S_q;
    uint32_t S_k;
    uint32_t D;
    uint32_t D_v;
    float scale;
    uint32_t maskType;  /* 0 = none, 1 = causal (top-left: key k visible to query q iff k <= q) */
};

/* ------------------------------------------------------------------------------------------
 * Launches.  All pointers are device pointers unless stated otherwise.
 * ---------------------------------------------------------------------------------------- */

/* z = x + y elementwise; dtype F32, F16 or BF16 (F16/BF16: one correctly rounded add).
 * Replaces elementwise_add_kernel (ops/elementwise_add/kernel/elementwise_add_kernel.cpp:88-97). */
int hc_elementwise_add_launch(const void* x, const void* y, void* z,
                              const struct elementwise_add_tiling_data* t, int dtype,
                              void* stream);

/* y = alpha * x + beta; dtype F32, F16 or BF16 (fp32 math).
 * Replaces axpy_scalar_affine_kernel (ops/axpy_scalar_affine/kernel/axpy_scalar_affine_kernel.cpp:64-72). */
int hc_axpy_scalar_affine_launch(const void* x, void* y,
                                 const struct axpy_scalar_affine_tiling_data* t, float alpha,
                                 float beta, int dtype, void* stream);

/* z[b,c,h,w] = x[b,c,h,w] * y[yb,c] + bias[c] (NCHW, yb = b if y_batch == B else 0);
 * x, y, bias, z share dtype F32, F16 or BF16 (fp32 math).
 * Replaces broadcast_binary_kernel (ops/broadcast_binary/kernel/broadcast_binary_kernel.cpp:122-134). */
int hc_broadcast_binary_launch(const void* x, const void* y, const void* bias, void* z,
                               const struct broadcast_binary_tiling_data* t, int dtype,
                               void* stream);

/* y = GELU_tanh(x) or SiLU(x); dtype F32, F16 or BF16 (fp32 math).
 * Replaces activation_gelu_silu_kernel (ops/activation_gelu_silu/kernel/activation_gelu_silu_kernel.cpp:145-155). */
int hc_activation_gelu_silu_launch(const void* x, void* y,
                                   const struct activation_gelu_silu_tiling_data* t, int dtype,
                                   void* stream);

/* out[r] = sum_k x[r,k], x dtype F32, F16 or BF16, out always F32 (fp32 accumulation).
 * Replaces reduce_sum_lastdim_kernel (ops/reduce_sum_lastdim/kernel/reduce_sum_lastdim_kernel.cpp:92-102). */
int hc_reduce_sum_lastdim_launch(const void* x, float* out,
                                 const struct reduce_sum_lastdim_tiling_data* t, int dtype,
                                 void* stream);

/* Index permutation (bit-exact): mode 0 2D transpose, 1 NCHW->NHWC, 2 NHWC->NCHW.
 * Any dtype; only the element size matters.  src and dst must not overlap.
 * Replaces transpose_2d_4d_kernel (ops/transpose_2d_4d/kernel/transpose_2d_4d_kernel.cpp:237-256). */
int hc_transpose_2d_4d_launch(const void* src, void* dst,
                              const struct transpose_2d_4d_tiling_data* t, int dtype,
                              void* stream);

/* y = (x - mean) / sqrt(var + eps) * gamma + beta over the last dim (two-pass, fp32 stats).
 * x, y dtype F32 or BF16 or F16; gamma, beta always F32.
 * Replaces layer_norm_kernel (ops/layer_norm/kernel/layer_norm_kernel.cpp:184-196). */
int hc_layer_norm_launch(const void* x, const float* gamma, const float* beta, void* y,
                         const struct layer_norm_tiling_data* t, int dtype, void* stream);

/* RMSNorm over each row of H elements (y = x / sqrt(mean(x^2) + eps) * weight), then RoPE on
 * the first rotaryDim elements with cos/sin tables of shape [S, rotaryDim/2] (fp32) indexed by
 * the row's sequence position s = (row / heads) % S.
 *   rope_style 0: interleaved pairs (2d, 2d+1), as the reference golden
 *                 (ops/rms_norm_rope_fused/golden/rms_norm_rope_fused_golden.cpp:40-51);
 *   rope_style 1: rotate-half pairs (d, d + rotaryDim/2).
 * x/out dtype F32, BF16 or F16; weight, cos, sin F32.  heads = 1 gives the reference's
 * [B, S, H] layout; heads = Hh gives [B, S, Hh, H].
 * Replaces rms_norm_rope_fused_kernel (ops/rms_norm_rope_fused/kernel/rms_norm_rope_fused_kernel.cpp:225-237). */
int hc_rms_norm_rope_fused_launch(const void* x, const float* weight, const float* cos_table,
                                  const float* sin_table, void* out,
                                  const struct rms_norm_rope_fused_tiling_data* t,
                                  uint32_t heads, uint32_t rope_style, int dtype, void* stream);

/* C[M,N] = A[M,K] . B[K,N] + bias[N] (row-major; bias may be NULL), fp32 accumulation.
 * dtype BF16 or F16 (A, B, bias, C all of that type) -> tcgen05 tensor-core kernel;
 * dtype F32 -> fp32 SIMT kernel.
 * Replaces matmul_bias_kernel (ops/matmul_bias/kernel/matmul_bias_kernel.cpp:181-193). */
int hc_matmul_bias_launch(const void* A, const void* B, const void* bias, void* C,
                          const struct matmul_bias_tiling_data* t, int dtype, void* stream);

/* O = softmax(Q K^T * scale [+ causal mask]) V with Q [B,H,S_q,D], K [B,H,S_k,D],
 * V [B,H,S_k,D_v], O [B,H,S_q,D_v] contiguous; optional lse [B,H,S_q] fp32 = natural-log
 * log-sum-exp of the scaled, masked scores (may be NULL).
 * dtype BF16 or F16 with D and D_v each 64 or 128 (16-byte aligned buffers) -> tcgen05/TMEM
 * kernel; any other D/D_v (<= 256) or dtype F32 -> SIMT kernel.  S_k >= 1 required.
 * Replaces flash_attention_fwd_fused_kernel
 * (ops/flash_attention_fwd_fused/kernel/flash_attention_fwd_fused_kernel.cpp:319-333). */
int hc_flash_attention_fwd_fused_launch(const void* q, const void* k, const void* v, void* o,
                                        float* lse,
                                        const struct flash_attention_fwd_fused_tiling_data* t,
                                        int dtype, void* stream);

/* Grouped-query form of the same kernel: K and V hold kv_heads heads ([B,kv_heads,S_k,D] and
 * [B,kv_heads,S_k,D_v]), and query head h reads K/V head h / (H / kv_heads).  kv_heads must
 * divide H (HC_ERR_INVALID otherwise, checked before any device work); kv_heads == H is
 * hc_flash_attention_fwd_fused_launch.  No counterpart in the reference: its tiling record has
 * no K/V head count, so this is an extra entry point rather than a change to the reference's
 * launch ABI. */
int hc_flash_attention_fwd_fused_gqa_launch(const void* q, const void* k, const void* v, void* o,
                                            float* lse,
                                            const struct flash_attention_fwd_fused_tiling_data* t,
                                            uint32_t kv_heads, int dtype, void* stream);

/* End-to-end variant with HOST buffers (pinned or pageable): copies q/k/v in, runs the kernel
 * and copies o/lse out, pipelined over chunks of (b,h) heads so that transfers overlap the
 * kernel.  `workspace` is a device buffer of at least
 * hc_flash_attention_fwd_fused_host_workspace_size() bytes owned by the caller.  Returns after
 * the outputs are in host memory; after an error it returns only once the work it had queued
 * is finished, so the workspace and host buffers may be reused at once.  Calls on one device
 * are serialised inside the library (its internal streams and events are per device).  Mirrors
 * the reference runner's host-pointer contract
 * (ops/flash_attention_fwd_fused/runner/flash_attention_fwd_fused_runner.hpp:9-18). */
int hc_flash_attention_fwd_fused_host_workspace_size(
    const struct flash_attention_fwd_fused_tiling_data* t, int dtype, size_t* bytes);
int hc_flash_attention_fwd_fused_host(const void* h_q, const void* h_k, const void* h_v,
                                      void* h_o, float* h_lse,
                                      const struct flash_attention_fwd_fused_tiling_data* t,
                                      int dtype, void* workspace, size_t workspace_bytes,
                                      void* stream);

/* Allocation-free variant of hc_flash_attention_fwd_fused_host (no counterpart in the reference):
 * the device staging memory is a fixed scratch array inside this library, so the call allocates
 * no device memory (no cudaMalloc / cudaFree, no allocating library routine) and creates no
 * streams or events.  It is meant for callers that cannot allocate on this path, such as a
 * serving loop whose device memory is fully reserved by its own pool, where an allocation could
 * fail or would synchronise the device.  Copies and kernels run in order on `stream`, one chunk
 * of whole heads at a time (no copy/compute overlap); returns when h_o / h_lse hold the result.
 *   Limit: hc_flash_attention_fwd_fused_host_noalloc_limit() bytes (64 MiB) of staging per
 *   device; a head whose q, k, v, o and lse do not fit, and every tiling the kernel would
 *   reject, is refused before any device work.
 *   The scratch array is part of the library's device image: each device the library is loaded
 *   on holds those 64 MiB until the process exits, whether or not this entry point is called.
 *   The first call on a device does one-time setup (the scratch's address is looked up with
 *   cudaGetSymbolAddress, the kernel sets its attributes): make it before any stream capture.
 *   The call waits for `stream` to drain before it returns, also after an error once a copy
 *   was queued.  Nothing in the scratch needs to start at zero.  Calls that overlap in time on
 *   one device (other threads or streams) race on the single scratch array and must be
 *   serialised. */
int hc_flash_attention_fwd_fused_host_noalloc(const void* h_q, const void* h_k, const void* h_v, void* h_o,
                                              float* h_lse,
                                              const struct flash_attention_fwd_fused_tiling_data* t,
                                              int dtype, void* stream);
size_t hc_flash_attention_fwd_fused_host_noalloc_limit(void);

/* Backward of hc_flash_attention_fwd_fused_launch (no counterpart in the reference: its ladder is
 * forward only).  From q, k, v, the forward's o and lse (natural log) and the output gradient
 * dO [B,H,S_q,D_v], writes dq [B,H,S_q,D], dk [B,H,S_k,D], dv [B,H,S_k,D_v] (all in `dtype`, every
 * element written) and delta [B,H,S_q] fp32 = rowsum(dO * o), a caller-owned buffer the second
 * kernel reads:  P = exp(S * scale - lse), dv = P^T dO, dS = P * (dO V^T - delta),
 * dq = scale * dS K, dk = scale * dS^T Q.  Same tiling record and checks as the forward
 * (K/V have H heads; grouped-query heads are not supported here).
 * dtype BF16 or F16 with D = D_v = 64 or 128 (16-byte aligned buffers) -> two tcgen05/TMEM kernels
 * (dq+delta, then dk/dv), P and dS rounded to `dtype` for the tensor-core products as the
 * forward rounds P; other D/D_v (<= 256) or F32 -> SIMT kernels in fp32. */
int hc_flash_attention_bwd_launch(const void* q, const void* k, const void* v, const void* o,
                                  const void* dO, const float* lse, void* dq, void* dk, void* dv,
                                  float* delta, const struct flash_attention_fwd_fused_tiling_data* t,
                                  int dtype, void* stream);
/* Kernel selection of the last successful backward launch on this thread (1 tcgen05, 2 SIMT). */
int hc_flash_attention_bwd_last_path(void);

/* Kernel selection used by the last successful flash-attention / matmul_bias launch on this
 * thread: 1 = tcgen05/TMEM path, 2 = SIMT path, 3 = tcgen05 CTA-pair path (matmul_bias with
 * M >= 256: two SMs per 256x256 tile), 0 = none yet. */
int hc_flash_attention_last_path(void);
int hc_matmul_bias_last_path(void);

#ifdef __cplusplus
}
#endif

#endif /* HC_OPS_H */
