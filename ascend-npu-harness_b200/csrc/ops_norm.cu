// layer_norm and rms_norm_rope_fused: row-wise normalisations, HBM-bound.
//
// A "row group" of TPR threads (8..1024, power of two) owns one row; each thread keeps VPT
// 16-byte packs of the row in registers, so HBM sees exactly one read and one write of x.
// A block processes RU rows per group per iteration with all loads issued before any
// reduction, which keeps enough bytes in flight per SM to saturate HBM for short rows
// (128-element RoPE heads) as well as long ones (4096-element LayerNorm rows).
//
// Arithmetic mirrors the reference goldens step by step (explicitly rounded fp32 ops, IEEE
// division and square root):
//   layer_norm          ops/layer_norm/golden/layer_norm_golden.cpp:15-39 (two-pass mean/var)
//   rms_norm_rope_fused ops/rms_norm_rope_fused/golden/rms_norm_rope_fused_golden.cpp:20-51
// The goldens accumulate sums in fp64; here the sums are fp32 shuffle trees, which is the
// only source of difference (well inside the bf16 tolerances).
#include <cuda_runtime.h>

#include "hc_device.cuh"
#include "hc_internal.h"

namespace hc {
namespace {

constexpr int kMaxVpt = 8;

enum class NormKind { kLayerNorm, kRmsRope };

struct NormArgs {
    const void* x;
    void* y;
    const float* gamma;  // LayerNorm gamma / RMSNorm weight
    const float* beta;   // LayerNorm only
    const float* cos_t;  // RoPE only, [S, rot/2]
    const float* sin_t;
    uint32_t rows;
    uint32_t H;          // row length
    uint32_t tpr;        // threads per row group
    float eps;
    uint32_t heads;      // rows per sequence position (RoPE)
    uint32_t S;
    uint32_t rot;        // rotary dim (even, <= H)
    uint32_t style;      // 0 interleaved, 1 rotate-half
};

template <int RU>
__device__ __forceinline__ void group_reduce(float (&v)[RU], uint32_t tpr, float* red) {
    if (tpr <= 32) {
#pragma unroll
        for (int r = 0; r < RU; ++r)
            for (uint32_t o = tpr >> 1; o > 0; o >>= 1) v[r] += __shfl_xor_sync(0xffffffffu, v[r], o);
        return;
    }
    // tpr > 32: warp trees, then the group's warps through shared memory.
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t wpg = tpr >> 5;                 // warps per group
    const uint32_t group = threadIdx.x / tpr;
#pragma unroll
    for (int r = 0; r < RU; ++r) {
        float s = warp_sum(v[r]);
        if (lane == 0) red[warp * RU + r] = s;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < RU; ++r) {
        float s = 0.f;
        for (uint32_t w = 0; w < wpg; ++w) s += red[(group * wpg + w) * RU + r];
        v[r] = s;
    }
    __syncthreads();
}

template <typename T, int VPT, int RU, NormKind KIND>
__global__ void __launch_bounds__(256) rownorm_kernel(NormArgs a) {
    constexpr int P = elem<T>::kPack;
    extern __shared__ float smem[];
    float* red = smem;                                   // (blockDim/32) * RU floats
    float* rope_buf = smem + (blockDim.x / 32) * RU;     // groups * RU * H floats (rotate-half only)

    const uint32_t tpr = a.tpr;
    const uint32_t groups = blockDim.x / tpr;
    const uint32_t group = threadIdx.x / tpr;
    const uint32_t gl = threadIdx.x % tpr;                 // lane within group
    const uint32_t packs = a.H / P;
    const uint64_t rows_per_iter = static_cast<uint64_t>(groups) * RU;
    const T* x = static_cast<const T*>(a.x);
    T* y = static_cast<T*>(a.y);
    const float inv_h = 1.0f / static_cast<float>(a.H);
    (void)inv_h;

    for (uint64_t base = static_cast<uint64_t>(blockIdx.x) * rows_per_iter; base < a.rows;
         base += static_cast<uint64_t>(gridDim.x) * rows_per_iter) {
        float xv[RU][VPT][P];
        // ---- loads (all rows of this iteration first) ----
#pragma unroll
        for (int r = 0; r < RU; ++r) {
            uint64_t row = base + group * RU + r;
#pragma unroll
            for (int v = 0; v < VPT; ++v) {
                uint32_t pi = v * tpr + gl;
                if (row < a.rows && pi < packs) {
                    pack<T> pk = ld_stream(reinterpret_cast<const pack<T>*>(x + row * a.H) + pi);
#pragma unroll
                    for (int e = 0; e < P; ++e) xv[r][v][e] = elem<T>::to_f(pk.v[e]);
                } else {
#pragma unroll
                    for (int e = 0; e < P; ++e) xv[r][v][e] = 0.f;
                }
            }
        }
        float scale_a[RU], shift_a[RU];
        if (KIND == NormKind::kLayerNorm) {
            float s[RU];
#pragma unroll
            for (int r = 0; r < RU; ++r) {
                s[r] = 0.f;
#pragma unroll
                for (int v = 0; v < VPT; ++v)
#pragma unroll
                    for (int e = 0; e < P; ++e) s[r] += xv[r][v][e];
            }
            group_reduce<RU>(s, tpr, red);
            float mean[RU];
#pragma unroll
            for (int r = 0; r < RU; ++r) mean[r] = __fdiv_rn(s[r], static_cast<float>(a.H));
#pragma unroll
            for (int r = 0; r < RU; ++r) {
                s[r] = 0.f;
#pragma unroll
                for (int v = 0; v < VPT; ++v) {
                    uint32_t pi = v * tpr + gl;
                    if (pi < packs) {
#pragma unroll
                        for (int e = 0; e < P; ++e) {
                            float d = __fsub_rn(xv[r][v][e], mean[r]);
                            s[r] = __fadd_rn(s[r], __fmul_rn(d, d));
                        }
                    }
                }
            }
            group_reduce<RU>(s, tpr, red);
#pragma unroll
            for (int r = 0; r < RU; ++r) {
                float var = __fdiv_rn(s[r], static_cast<float>(a.H));
                scale_a[r] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, a.eps)));  // inv_std
                shift_a[r] = mean[r];
            }
        } else {
            float s[RU];
#pragma unroll
            for (int r = 0; r < RU; ++r) {
                s[r] = 0.f;
#pragma unroll
                for (int v = 0; v < VPT; ++v)
#pragma unroll
                    for (int e = 0; e < P; ++e) s[r] = __fadd_rn(s[r], __fmul_rn(xv[r][v][e], xv[r][v][e]));
            }
            group_reduce<RU>(s, tpr, red);
#pragma unroll
            for (int r = 0; r < RU; ++r) {
                scale_a[r] = __fsqrt_rn(__fadd_rn(__fdiv_rn(s[r], static_cast<float>(a.H)), a.eps));  // rms
                shift_a[r] = 0.f;
            }
        }

        // ---- normalise ----
#pragma unroll
        for (int r = 0; r < RU; ++r) {
#pragma unroll
            for (int v = 0; v < VPT; ++v) {
                uint32_t pi = v * tpr + gl;
                if (pi >= packs) continue;
                uint32_t e0 = pi * P;
#pragma unroll
                for (int e = 0; e < P; ++e) {
                    float g = __ldg(a.gamma + e0 + e);
                    if (KIND == NormKind::kLayerNorm) {
                        float nrm = __fmul_rn(__fsub_rn(xv[r][v][e], shift_a[r]), scale_a[r]);
                        xv[r][v][e] = __fadd_rn(__fmul_rn(nrm, g), __ldg(a.beta + e0 + e));
                    } else {
                        xv[r][v][e] = __fmul_rn(__fdiv_rn(xv[r][v][e], scale_a[r]), g);
                    }
                }
            }
        }

        // ---- RoPE ----
        if (KIND == NormKind::kRmsRope && a.rot > 0) {
            const uint32_t half = a.rot / 2;
            if (a.style == 1) {
                // Rotate-half pairs (d, d + half) may live in different threads: exchange the
                // normalised row through shared memory.
#pragma unroll
                for (int r = 0; r < RU; ++r) {
                    float* buf = rope_buf + (static_cast<size_t>(group) * RU + r) * a.H;
#pragma unroll
                    for (int v = 0; v < VPT; ++v) {
                        uint32_t pi = v * tpr + gl;
                        if (pi >= packs) continue;
#pragma unroll
                        for (int e = 0; e < P; ++e) buf[pi * P + e] = xv[r][v][e];
                    }
                }
                if (tpr <= 32) __syncwarp(); else __syncthreads();
                // For tpr < 32 several groups share a warp; __syncwarp covers all of them.
            }
#pragma unroll
            for (int r = 0; r < RU; ++r) {
                uint64_t row = base + group * RU + r;
                if (row >= a.rows) continue;
                uint32_t s_pos = static_cast<uint32_t>((row / a.heads) % a.S);
                const float* cs = a.cos_t + static_cast<size_t>(s_pos) * half;
                const float* sn = a.sin_t + static_cast<size_t>(s_pos) * half;
                const float* buf = rope_buf + (static_cast<size_t>(group) * RU + r) * a.H;
#pragma unroll
                for (int v = 0; v < VPT; ++v) {
                    uint32_t pi = v * tpr + gl;
                    if (pi >= packs) continue;
                    float outv[P];
#pragma unroll
                    for (int e = 0; e < P; ++e) {
                        uint32_t d = pi * P + e;
                        float val = xv[r][v][e];
                        if (d < a.rot) {
                            if (a.style == 0) {
                                uint32_t i = d >> 1;
                                float c = __ldg(cs + i), z = __ldg(sn + i);
                                // pair partner sits in the same pack (P is even)
                                float other = (e & 1) ? xv[r][v][e - 1] : xv[r][v][e + 1];
                                if ((d & 1) == 0) val = __fsub_rn(__fmul_rn(val, c), __fmul_rn(other, z));
                                else val = __fadd_rn(__fmul_rn(other, z), __fmul_rn(val, c));
                            } else {
                                if (d < half) {
                                    float c = __ldg(cs + d), z = __ldg(sn + d);
                                    val = __fsub_rn(__fmul_rn(val, c), __fmul_rn(buf[d + half], z));
                                } else {
                                    uint32_t i = d - half;
                                    float c = __ldg(cs + i), z = __ldg(sn + i);
                                    val = __fadd_rn(__fmul_rn(buf[i], z), __fmul_rn(val, c));
                                }
                            }
                        }
                        outv[e] = val;
                    }
#pragma unroll
                    for (int e = 0; e < P; ++e) xv[r][v][e] = outv[e];
                }
            }
            if (a.style == 1) {
                if (tpr <= 32) __syncwarp(); else __syncthreads();
            }
        }

        // ---- stores ----
#pragma unroll
        for (int r = 0; r < RU; ++r) {
            uint64_t row = base + group * RU + r;
            if (row >= a.rows) continue;
#pragma unroll
            for (int v = 0; v < VPT; ++v) {
                uint32_t pi = v * tpr + gl;
                if (pi >= packs) continue;
                pack<T> pk;
#pragma unroll
                for (int e = 0; e < P; ++e) pk.v[e] = elem<T>::from_f(xv[r][v][e]);
                st_stream(reinterpret_cast<pack<T>*>(y + row * a.H) + pi, pk);
            }
        }
    }
}

// Scalar fallback (unaligned buffers or rows not a multiple of the pack): one block per row,
// three passes over the row (the row stays in L1/L2 between passes).
template <typename T, NormKind KIND>
__global__ void __launch_bounds__(256) rownorm_scalar_kernel(NormArgs a) {
    __shared__ float red[8];
    extern __shared__ float row_buf[];  // H floats
    const T* x = static_cast<const T*>(a.x);
    T* y = static_cast<T*>(a.y);
    for (uint64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
        const T* xr = x + row * a.H;
        float s = 0.f;
        for (uint32_t d = threadIdx.x; d < a.H; d += blockDim.x) {
            float v = elem<T>::to_f(xr[d]);
            row_buf[d] = v;
            s = (KIND == NormKind::kLayerNorm) ? __fadd_rn(s, v) : __fadd_rn(s, __fmul_rn(v, v));
        }
        auto block_sum = [&](float v) {
            v = warp_sum(v);
            if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
            __syncthreads();
            float t = 0.f;
            for (uint32_t w = 0; w < blockDim.x / 32; ++w) t += red[w];
            __syncthreads();
            return t;
        };
        s = block_sum(s);
        float scale, shift = 0.f;
        if (KIND == NormKind::kLayerNorm) {
            float mean = __fdiv_rn(s, static_cast<float>(a.H));
            float q = 0.f;
            for (uint32_t d = threadIdx.x; d < a.H; d += blockDim.x) {
                float dd = __fsub_rn(row_buf[d], mean);
                q = __fadd_rn(q, __fmul_rn(dd, dd));
            }
            q = block_sum(q);
            scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(q, static_cast<float>(a.H)), a.eps)));
            shift = mean;
        } else {
            scale = __fsqrt_rn(__fadd_rn(__fdiv_rn(s, static_cast<float>(a.H)), a.eps));
        }
        for (uint32_t d = threadIdx.x; d < a.H; d += blockDim.x) {
            float v = row_buf[d];
            if (KIND == NormKind::kLayerNorm)
                v = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v, shift), scale), a.gamma[d]), a.beta[d]);
            else
                v = __fmul_rn(__fdiv_rn(v, scale), a.gamma[d]);
            row_buf[d] = v;
        }
        __syncthreads();
        for (uint32_t d = threadIdx.x; d < a.H; d += blockDim.x) {
            float v = row_buf[d];
            if (KIND == NormKind::kRmsRope && d < a.rot) {
                uint32_t half = a.rot / 2;
                uint32_t s_pos = static_cast<uint32_t>((row / a.heads) % a.S);
                const float* cs = a.cos_t + static_cast<size_t>(s_pos) * half;
                const float* sn = a.sin_t + static_cast<size_t>(s_pos) * half;
                if (a.style == 0) {
                    uint32_t i = d >> 1;
                    if ((d & 1) == 0) v = __fsub_rn(__fmul_rn(v, cs[i]), __fmul_rn(row_buf[d + 1], sn[i]));
                    else v = __fadd_rn(__fmul_rn(row_buf[d - 1], sn[i]), __fmul_rn(v, cs[i]));
                } else {
                    if (d < half) v = __fsub_rn(__fmul_rn(v, cs[d]), __fmul_rn(row_buf[d + half], sn[d]));
                    else v = __fadd_rn(__fmul_rn(row_buf[d - half], sn[d - half]), __fmul_rn(v, cs[d - half]));
                }
            }
            y[row * a.H + d] = elem<T>::from_f(v);
        }
        __syncthreads();
    }
}

uint32_t next_pow2(uint32_t v) {
    uint32_t p = 1;
    while (p < v) p <<= 1;
    return p;
}

template <typename T, int VPT, NormKind KIND>
int launch_rownorm_vec(NormArgs a, uint32_t threads, cudaStream_t s) {
    constexpr int RU = (VPT <= 2) ? 2 : 1;
    uint32_t groups = threads / a.tpr;
    size_t smem = (threads / 32) * RU * sizeof(float);
    if (KIND == NormKind::kRmsRope && a.style == 1) smem += static_cast<size_t>(groups) * RU * a.H * sizeof(float);
    if (smem > 48 * 1024) {
        if (cudaFuncSetAttribute(rownorm_kernel<T, VPT, RU, KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem)) != cudaSuccess)
            return cuda_fail(cudaGetLastError(), "cudaFuncSetAttribute(rownorm)");
    }
    uint64_t iters = (a.rows + static_cast<uint64_t>(groups) * RU - 1) / (static_cast<uint64_t>(groups) * RU);
    uint64_t cap = static_cast<uint64_t>(sm_count()) * (2048 / threads);
    int blocks = static_cast<int>(iters < cap ? iters : cap);
    rownorm_kernel<T, VPT, RU, KIND><<<blocks, threads, smem, s>>>(a);
    return check_launch(KIND == NormKind::kLayerNorm ? "layer_norm" : "rms_norm_rope_fused");
}

template <typename T, NormKind KIND>
int launch_rownorm(NormArgs a, void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    constexpr uint32_t P = elem<T>::kPack;
    const uint32_t packs = a.H / P;
    bool vec = (a.H % P == 0) && aligned16(a.x) && aligned16(a.y) && packs <= 1024 * kMaxVpt;
    if (vec) {
        // Aim for 4 packs per thread; groups of at least 8 threads (tiny rows) and at most 1024.
        uint32_t tpr = next_pow2((packs + 3) / 4);
        if (tpr < 8) tpr = 8;
        if (tpr > 1024) tpr = 1024;
        uint32_t vpt = next_pow2((packs + tpr - 1) / tpr);
        if (vpt == 0) vpt = 1;
        a.tpr = tpr;
        uint32_t threads = tpr < 256 ? 256 : tpr;
        switch (vpt) {
            case 1: return launch_rownorm_vec<T, 1, KIND>(a, threads, s);
            case 2: return launch_rownorm_vec<T, 2, KIND>(a, threads, s);
            case 4: return launch_rownorm_vec<T, 4, KIND>(a, threads, s);
            case 8: return launch_rownorm_vec<T, 8, KIND>(a, threads, s);
            default: break;
        }
    }
    size_t smem = static_cast<size_t>(a.H) * sizeof(float);
    if (smem > 200 * 1024) return fail(HC_ERR_UNSUPPORTED, "row length %u too long for the scalar row kernel", a.H);
    if (smem > 48 * 1024) {
        if (cudaFuncSetAttribute(rownorm_scalar_kernel<T, KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem)) != cudaSuccess)
            return cuda_fail(cudaGetLastError(), "cudaFuncSetAttribute(rownorm_scalar)");
    }
    uint64_t cap = static_cast<uint64_t>(sm_count()) * 8;
    int blocks = static_cast<int>(a.rows < cap ? a.rows : cap);
    rownorm_scalar_kernel<T, KIND><<<blocks, 256, smem, s>>>(a);
    return check_launch(KIND == NormKind::kLayerNorm ? "layer_norm(scalar)" : "rms_norm_rope_fused(scalar)");
}

template <NormKind KIND>
int dispatch_rownorm(int dtype, const NormArgs& a, void* stream, const char* name) {
    switch (dtype) {
        case HC_DTYPE_F32: return launch_rownorm<float, KIND>(a, stream);
        case HC_DTYPE_F16: return launch_rownorm<f16_t, KIND>(a, stream);
        case HC_DTYPE_BF16: return launch_rownorm<bf16_t, KIND>(a, stream);
        default: return fail(HC_ERR_UNSUPPORTED, "%s: dtype %d not supported (F32, F16, BF16)", name, dtype);
    }
}

}  // namespace
}  // namespace hc

using namespace hc;

extern "C" int hc_layer_norm_launch(const void* x, const float* gamma, const float* beta, void* y,
                                    const layer_norm_tiling_data* t, int dtype, void* stream) {
    if (!t) return fail(HC_ERR_INVALID, "layer_norm: null tiling");
    if (t->rows == 0) return ok();
    if (!x || !gamma || !beta || !y || t->lastDim == 0) return fail(HC_ERR_INVALID, "layer_norm: null pointer or zero lastDim");
    if (fault_hit("launch")) return fail(HC_ERR_INJECTED, "layer_norm: injected launch failure");
    NormArgs a{};
    a.x = x; a.y = y; a.gamma = gamma; a.beta = beta;
    a.rows = t->rows; a.H = t->lastDim; a.eps = t->eps;
    a.heads = 1; a.S = 1;
    return dispatch_rownorm<NormKind::kLayerNorm>(dtype, a, stream, "layer_norm");
}

extern "C" int hc_rms_norm_rope_fused_launch(const void* x, const float* weight, const float* cos_table,
                                             const float* sin_table, void* out, const rms_norm_rope_fused_tiling_data* t,
                                             uint32_t heads, uint32_t rope_style, int dtype, void* stream) {
    if (!t) return fail(HC_ERR_INVALID, "rms_norm_rope_fused: null tiling");
    if (heads == 0) return fail(HC_ERR_INVALID, "rms_norm_rope_fused: heads must be >= 1");
    if (rope_style > 1) return fail(HC_ERR_INVALID, "rms_norm_rope_fused: rope_style %u (0 interleaved, 1 rotate-half)", rope_style);
    if (t->H == 0) return fail(HC_ERR_INVALID, "rms_norm_rope_fused: H == 0");
    if (t->rotaryDim > t->H || (t->rotaryDim & 1)) return fail(HC_ERR_INVALID, "rms_norm_rope_fused: rotaryDim %u must be even and <= H %u", t->rotaryDim, t->H);
    uint64_t rows = static_cast<uint64_t>(t->B) * t->S * heads;
    if (rows == 0) return ok();
    if (rows > 0xffffffffull) return fail(HC_ERR_UNSUPPORTED, "rms_norm_rope_fused: too many rows");
    if (!x || !weight || !out || (t->rotaryDim && (!cos_table || !sin_table)))
        return fail(HC_ERR_INVALID, "rms_norm_rope_fused: null pointer");
    if (fault_hit("launch")) return fail(HC_ERR_INJECTED, "rms_norm_rope_fused: injected launch failure");
    NormArgs a{};
    a.x = x; a.y = out; a.gamma = weight; a.beta = nullptr; a.cos_t = cos_table; a.sin_t = sin_table;
    a.rows = static_cast<uint32_t>(rows); a.H = t->H; a.eps = t->eps;
    a.heads = heads; a.S = t->S; a.rot = t->rotaryDim; a.style = rope_style;
    return dispatch_rownorm<NormKind::kRmsRope>(dtype, a, stream, "rms_norm_rope_fused");
}
