// layer_norm and rms_norm_rope_fused: row-wise normalisations, HBM-bound.
//
// Two kernel shapes; both read every element from HBM once and write it once.
//
// Row-stream kernel (short and medium rows; all RMSNorm+RoPE shapes), one persistent CTA per SM,
// 800 threads:
//   * a producer thread copies tiles of whole consecutive rows from HBM into a ring of
//     shared-memory stages with single bulk TMA copies (cp.async.bulk, completion on an mbarrier),
//     keeping up to ~190 KB per SM in flight without holding rows in registers;
//   * up to six consumer groups of four warps take turns on the stages (group g takes this CTA's
//     tiles g, g+groups, ...); inside a tile a group of G = 8/16/32 lanes owns one row, reduces it
//     with shuffles, then normalises it from shared memory and leaves with 16-byte streaming
//     stores; each consumer warp releases the stage through an mbarrier when its rows are done;
//   * row processing is specialised at compile time where the shape allows: rows of exactly
//     32*KPL packs (unrolled LayerNorm), and rotate-half RoPE over the whole row, where lane gl
//     holds pack gl and its rotation partner pack gl+G (no data from other lanes, weights kept in
//     registers); both do their arithmetic on f32x2 pairs.  A generic loop handles the rest.
//
// Direct LayerNorm kernel (rows of 1024*KPL 16-bit / 512*KPL fp32 elements): a 128-thread group
// owns whole rows, keeps its share of the current row in registers and issues the streaming loads
// of its next row before working on the current one; one-pass shifted statistics with an exact
// fallback pass, combined across the group's warps through shared memory and a named barrier.
//
// Arithmetic follows the reference goldens step by step:
//   layer_norm          ops/layer_norm/golden/layer_norm_golden.cpp:15-39 (two-pass mean/var,
//                       inv_std = 1/sqrt(var+eps), y = (x-mean)*inv_std*gamma + beta); the
//                       statistics use correctly rounded fp32 adds, division and square root;
//   rms_norm_rope_fused ops/rms_norm_rope_fused/golden/rms_norm_rope_fused_golden.cpp:20-51
//                       (rms = sqrt(mean(x^2)+eps), y = x/rms*w, then the rotation).
// Differences from the goldens: sums are fp32 (per-lane partial sums, then a shuffle tree)
// instead of sequential fp64 -- for LayerNorm taken over deviations from the row's first element,
// which keeps the mean accurate for rows near a large constant; x/rms is computed as x*(1/rms);
// per-element products may be fused into multiply-adds and RMS uses rsqrtf (a few ulp of fp32,
// far below the 16-bit output rounding): an IEEE division per element would make the kernel
// instruction-bound instead of HBM-bound.  The scalar fallback kernel keeps every fp32 operation
// explicitly rounded.
//
// Rows that are not a multiple of 16 bytes, or unaligned buffers, use that simple scalar kernel.
// Waits are bounded like the tensor-core kernels'; an expired wait is reported through
// hc_check_device_error().
#include <cuda_runtime.h>

#include <mutex>

#include "hc_device.cuh"
#include "hc_internal.h"
#include "sm100.cuh"

namespace hc {
namespace {

using namespace sm100;

enum class NormKind { kLayerNorm, kRmsRope };

// Consumers: kGroups groups of kGroupWarps warps; group g takes this CTA's tiles i = g, g+kGroups,
// ..., so two tiles are being normalised while further stages are in flight.
// The number of groups actually used (a.groups <= kGroups) is chosen at launch so that every
// active group has a tile to work on and at least one more stage is being filled.
constexpr uint32_t kGroupWarps = 4;
constexpr uint32_t kGroups = 6;
constexpr uint32_t kConsumerWarps = kGroupWarps * kGroups;
constexpr uint32_t kThreads = (kConsumerWarps + 1) * 32;  // + one producer warp
constexpr uint32_t kMaxStages = 12;
constexpr uint32_t kSmemBudget = 200 * 1024;

__device__ uint32_t g_norm_error_word;

struct NormArgs {
    const void* x;
    void* y;
    const float* gamma;  // LayerNorm gamma / RMSNorm weight
    const float* beta;   // LayerNorm only
    const float* cos_t;  // RoPE only, [S, rot/2]
    const float* sin_t;
    uint32_t rows;
    uint32_t H;          // row length (elements)
    float eps;
    uint32_t heads;      // rows per sequence position (RoPE)
    uint32_t S;
    uint32_t rot;        // rotary dim (even, <= H)
    uint32_t style;      // 0 interleaved, 1 rotate-half
    uint32_t tile_rows;  // rows per shared-memory stage
    uint32_t stages;
    uint32_t tile_bytes;       // tile_rows * H * sizeof(T), multiple of 16
    uint32_t param_floats;     // floats of parameters staged in shared memory
    uint32_t param_stride;     // floats per staged parameter vector (lane-transposed, padded)
    uint32_t vec_rope;         // 1: rotary packs never straddle the rotary boundary or the halves
    float inv_h;               // 1/H
    uint32_t groups;           // consumer groups in use (<= kGroups)
    uint32_t xor_partner;      // 1: one pack per lane, rotate-half partner on lane gl ^ G/2
    FastDiv div_heads, div_S;  // row -> sequence position (row / heads) % S

    __device__ __forceinline__ uint32_t pos_of_row(uint32_t row) const { return div_S.mod(div_heads.div(row)); }
};

struct RingBars {
    uint64_t full[kMaxStages], empty[kMaxStages];
};

template <int G>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
    for (int o = G / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Reads one 16-byte pack from shared memory with a single 128-bit load (a member-wise copy of the
// 16-bit struct would become eight 2-byte loads, 4-way bank-conflicted across the warp).
template <typename T>
__device__ __forceinline__ void unpack_f(const pack<T>& p, float* f) {
    const uint4 raw = *reinterpret_cast<const uint4*>(&p);
    const pack<T>& q = *reinterpret_cast<const pack<T>*>(&raw);
#pragma unroll
    for (int e = 0; e < elem<T>::kPack; ++e) f[e] = elem<T>::to_f(q.v[e]);
}

// Shared-memory layout of a staged parameter vector, transposed by lane: lane gl of a row group
// always handles packs k = gl + G*i, so the four parameters of quad q of pack k are stored at
// float index ((i * P/4 + q) * G + gl) * 4.  Consecutive lanes then read consecutive 16-byte
// slots (no bank conflicts), where the natural layout would put them 4*P bytes apart.
template <int P, int G>
__device__ __forceinline__ uint32_t param_slot(uint32_t k, uint32_t q) {
    return ((k / G * (P / 4) + q) * G + k % G) * 4;
}

template <int P, int G>
__device__ __forceinline__ void load_params(const float* base, uint32_t k, float* out) {
#pragma unroll
    for (int q = 0; q < P / 4; ++q) {
        const float4 v = *reinterpret_cast<const float4*>(base + param_slot<P, G>(k, q));
        out[4 * q] = v.x; out[4 * q + 1] = v.y; out[4 * q + 2] = v.z; out[4 * q + 3] = v.w;
    }
}

template <int N>
__device__ __forceinline__ void ldg_f32(const float* p, float* out) {
    if (N % 4 == 0) {
#pragma unroll
        for (int i = 0; i < N; i += 4) {
            const float4 v = __ldg(reinterpret_cast<const float4*>(p + i));
            out[i] = v.x; out[i + 1] = v.y; out[i + 2] = v.z; out[i + 3] = v.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < N; i += 2) {
            const float2 v = __ldg(reinterpret_cast<const float2*>(p + i));
            out[i] = v.x; out[i + 1] = v.y;
        }
    }
}

// Processes one row held in shared memory with the G lanes of a row group.  Every lane of the warp
// calls it the same number of times (the shuffles use the full mask); groups without a row of
// their own pass valid = false and only take part in the shuffles.
template <typename T, NormKind KIND, int G>
__device__ __forceinline__ void process_row(const NormArgs& a, const pack<T>* srow, const float* params, uint64_t row,
                                            uint32_t gl, bool valid) {
    constexpr int P = elem<T>::kPack;
    const uint32_t packs = valid ? a.H / P : 0u;
    const float invH = 1.0f / static_cast<float>(a.H);
    (void)invH;
    // ---- pass 1 (and 2 for LayerNorm): statistics from shared memory ----
    const float K = (KIND == NormKind::kLayerNorm) ? elem<T>::to_f(srow[0].v[0]) : 0.f;  // LayerNorm shift
    float s = 0.f;
    for (uint32_t k = gl; k < packs; k += G) {
        float f[P];
        unpack_f<T>(srow[k], f);
#pragma unroll
        for (int e = 0; e < P; ++e)
            s = (KIND == NormKind::kLayerNorm) ? __fadd_rn(s, __fsub_rn(f[e], K)) : fmaf(f[e], f[e], s);
    }
    s = group_sum<G>(s);
    float mul, sub = 0.f;
    if (KIND == NormKind::kLayerNorm) {
        const float mean = __fadd_rn(K, __fdiv_rn(s, static_cast<float>(a.H)));
        float q = 0.f;
        for (uint32_t k = gl; k < packs; k += G) {
            float f[P];
            unpack_f<T>(srow[k], f);
#pragma unroll
            for (int e = 0; e < P; ++e) {
                const float d = __fsub_rn(f[e], mean);
                q = __fadd_rn(q, __fmul_rn(d, d));
            }
        }
        q = group_sum<G>(q);
        mul = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(q, static_cast<float>(a.H)), a.eps)));  // inv_std
        sub = mean;
    } else {
        // 1/rms with the hardware reciprocal square root: rows are short (128 elements in the
        // RoPE configuration), so IEEE division and square root per row would cost as many
        // instructions as the row itself.  Error <= 2 ulp, far inside the tolerances.
        mul = rsqrtf(fmaf(s, a.inv_h, a.eps));
    }
    // ---- last pass: normalise (+ RoPE) and store ----
    const uint32_t half = a.rot / 2;
    const float* cs = nullptr;
    const float* sn = nullptr;
    if (KIND == NormKind::kRmsRope) {
        const uint32_t s_pos = valid ? a.pos_of_row(static_cast<uint32_t>(row)) : 0u;
        cs = a.cos_t + static_cast<size_t>(s_pos) * half;
        sn = a.sin_t + static_cast<size_t>(s_pos) * half;
        if (a.xor_partner) {
            // One pack per lane and rotate-half over the whole row: the partner of lane gl's pack
            // is lane gl ^ G/2's pack, so the normalised partner values come over a shuffle
            // (every lane of the warp executes this branch: the flag is kernel-wide).
            float f[P], g[P], c[P], z[P], out[P];
            unpack_f<T>(srow[gl], f);
            load_params<P, G>(params, gl, g);
            const bool first = gl < G / 2;
            const uint32_t i0 = (first ? gl : gl - G / 2) * P;
            ldg_f32<P>(cs + i0, c);
            ldg_f32<P>(sn + i0, z);
#pragma unroll
            for (int e = 0; e < P; ++e) out[e] = f[e] * mul * g[e];
            const float zs = first ? -1.f : 1.f;  // first half: y c - p z; second: p z + y c
#pragma unroll
            for (int e = 0; e < P; ++e) {
                const float partner = __shfl_xor_sync(0xffffffffu, out[e], G / 2);
                out[e] = fmaf(out[e], c[e], zs * partner * z[e]);
            }
            if (valid) {
                T* yrow = static_cast<T*>(a.y) + row * a.H;
                st_stream(reinterpret_cast<pack<T>*>(yrow) + gl, pack_from_f<T>(out));
            }
            return;
        }
    }
    if (!valid) return;
    T* yrow = static_cast<T*>(a.y) + row * a.H;
    for (uint32_t k = gl; k < packs; k += G) {
        const uint32_t d0 = k * P;
        float f[P], g[P];
        unpack_f<T>(srow[k], f);
        load_params<P, G>(params, k, g);
        float out[P];
        if (KIND == NormKind::kLayerNorm) {
            float b[P];
            load_params<P, G>(params + a.param_stride, k, b);
#pragma unroll
            for (int e = 0; e < P; ++e) out[e] = fmaf((f[e] - sub) * mul, g[e], b[e]);
        } else {
#pragma unroll
            for (int e = 0; e < P; ++e) out[e] = __fmul_rn(__fmul_rn(f[e], mul), g[e]);
            if (a.vec_rope && d0 < a.rot) {
                // Whole pack inside the rotary part, tables read as vectors.
                if (a.style == 0) {
                    float c[P / 2], z[P / 2];
                    ldg_f32<P / 2>(cs + d0 / 2, c);
                    ldg_f32<P / 2>(sn + d0 / 2, z);
#pragma unroll
                    for (int e = 0; e < P; e += 2) {
                        const float ye = out[e], yo = out[e + 1];
                        out[e] = fmaf(ye, c[e / 2], -yo * z[e / 2]);
                        out[e + 1] = fmaf(ye, z[e / 2], yo * c[e / 2]);
                    }
                } else {
                    const bool first = d0 < half;
                    const uint32_t kp = first ? k + half / P : k - half / P;  // partner pack
                    float fp[P], gp[P], c[P], z[P];
                    unpack_f<T>(srow[kp], fp);
                    load_params<P, G>(params, kp, gp);
                    ldg_f32<P>(cs + (first ? d0 : d0 - half), c);
                    ldg_f32<P>(sn + (first ? d0 : d0 - half), z);
                    const float zs = first ? -1.f : 1.f;  // first half: y c - p z; second: p z + y c
#pragma unroll
                    for (int e = 0; e < P; ++e) {
                        const float partner = fp[e] * mul * gp[e];
                        out[e] = fmaf(out[e], c[e], zs * partner * z[e]);
                    }
                }
            } else if (d0 < a.rot) {
                if (a.style == 0) {
                    // interleaved pairs (2i, 2i+1); a pack starts on an even column
#pragma unroll
                    for (int e = 0; e < P; e += 2) {
                        const uint32_t d = d0 + e;
                        if (d < a.rot) {
                            const float c = __ldg(cs + d / 2), z = __ldg(sn + d / 2);
                            const float ye = out[e], yo = out[e + 1];
                            out[e] = __fsub_rn(__fmul_rn(ye, c), __fmul_rn(yo, z));
                            out[e + 1] = __fadd_rn(__fmul_rn(ye, z), __fmul_rn(yo, c));
                        }
                    }
                } else {
                    // rotate-half pairs (d, d + half): the partner is read from the staged row
                    const T* xs = reinterpret_cast<const T*>(srow);
#pragma unroll
                    for (int e = 0; e < P; ++e) {
                        const uint32_t d = d0 + e;
                        if (d < a.rot) {
                            const bool first = d < half;
                            const uint32_t i = first ? d : d - half;
                            const uint32_t pd = first ? d + half : d - half;
                            const float wp = params[param_slot<P, G>(pd / P, (pd % P) / 4) + pd % 4];
                            const float partner = __fmul_rn(__fmul_rn(elem<T>::to_f(xs[pd]), mul), wp);
                            const float c = __ldg(cs + i), z = __ldg(sn + i);
                            out[e] = first ? __fsub_rn(__fmul_rn(out[e], c), __fmul_rn(partner, z))
                                           : __fadd_rn(__fmul_rn(partner, z), __fmul_rn(out[e], c));
                        }
                    }
                }
            }
        }
        st_stream(reinterpret_cast<pack<T>*>(yrow) + k, pack_from_f<T>(out));
    }
}

// ---- 16-byte packs as float2 pairs (element 2i in .x, 2i+1 in .y) ----
template <typename T>
struct Pk;
template <>
struct Pk<bf16_t> {
    static constexpr int N2 = 4;
    __device__ static void unpack(const uint4& r, float2* f) {
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) f[i] = make_float2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xffff0000u));
    }
    __device__ static uint4 pack(const float2* f) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            __nv_bfloat162 h = __float22bfloat162_rn(f[i]);
            w[i] = *reinterpret_cast<uint32_t*>(&h);
        }
        return make_uint4(w[0], w[1], w[2], w[3]);
    }
};
template <>
struct Pk<f16_t> {
    static constexpr int N2 = 4;
    __device__ static void unpack(const uint4& r, float2* f) {
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) f[i] = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    }
    __device__ static uint4 pack(const float2* f) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            __half2 h = __float22half2_rn(f[i]);
            w[i] = *reinterpret_cast<uint32_t*>(&h);
        }
        return make_uint4(w[0], w[1], w[2], w[3]);
    }
};
template <>
struct Pk<float> {
    static constexpr int N2 = 2;
    __device__ static void unpack(const uint4& r, float2* f) {
        f[0] = make_float2(__uint_as_float(r.x), __uint_as_float(r.y));
        f[1] = make_float2(__uint_as_float(r.z), __uint_as_float(r.w));
    }
    __device__ static uint4 pack(const float2* f) {
        return make_uint4(__float_as_uint(f[0].x), __float_as_uint(f[0].y), __float_as_uint(f[1].x),
                          __float_as_uint(f[1].y));
    }
};

// Shift for the LayerNorm mean: the row's first element.  The mean is computed as
// K + sum(x - K) / H, so the fp32 partial sums hold deviations from a value of the row instead of
// the raw values: the error of the mean then stays a small fraction of the row's spread even when
// |mean| >> spread (rows near a large constant), where a plain fp32 sum of x would lose the mean.
// (The reference golden sums in fp64, layer_norm_golden.cpp:19-23.)
template <typename T>
__device__ __forceinline__ float row_shift(const T* row) {
    return elem<T>::to_f(row[0]);
}

// Row processors specialised at compile time for rows of exactly G * KPL packs: lane gl of the
// row group owns packs gl + G*j, every loop is unrolled and the arithmetic runs on f32x2 pairs
// (one FFMA2/FADD2/FMUL2 per two elements).  The generic process_row above handles every
// other shape.

// LayerNorm: mean, centred sum of squares, normalise -- three passes over the staged row.  The
// pass loops are unrolled only 4 / 2 deep: at 800 threads a thread has 80 registers, and fully
// unrolled passes would hoist every load of the row and spill.
template <typename T, int G, int KPL>
__device__ __forceinline__ void ln_row_fast(const NormArgs& a, const uint4* srow, const float* params, uint64_t row,
                                            uint32_t gl, bool valid) {
    constexpr int N2 = Pk<T>::N2, P = 2 * N2;
    // Sum of deviations from the row's first element (see row_shift).
    const float K = row_shift(reinterpret_cast<const T*>(srow));
    const float2 nk = make_float2(-K, -K);
    float2 acc0 = make_float2(0.f, 0.f), acc1 = acc0;
#pragma unroll(KPL > 4 ? 4 : 2)
    for (int j = 0; j < KPL; ++j) {
        float2 f[N2];
        Pk<T>::unpack(srow[gl + G * j], f);
#pragma unroll
        for (int i = 0; i < N2; ++i) {
            if (i & 1) acc1 = __fadd2_rn(acc1, __fadd2_rn(f[i], nk));
            else acc0 = __fadd2_rn(acc0, __fadd2_rn(f[i], nk));
        }
    }
    const float mean =
        __fadd_rn(K, __fdiv_rn(group_sum<G>((acc0.x + acc0.y) + (acc1.x + acc1.y)), static_cast<float>(a.H)));
    const float2 nmean = make_float2(-mean, -mean);
    acc0 = acc1 = make_float2(0.f, 0.f);
#pragma unroll(KPL > 4 ? 4 : 2)
    for (int j = 0; j < KPL; ++j) {
        float2 f[N2];
        Pk<T>::unpack(srow[gl + G * j], f);
#pragma unroll
        for (int i = 0; i < N2; ++i) {
            const float2 d = __fadd2_rn(f[i], nmean);
            if (i & 1) acc1 = __ffma2_rn(d, d, acc1);
            else acc0 = __ffma2_rn(d, d, acc0);
        }
    }
    const float q = group_sum<G>((acc0.x + acc0.y) + (acc1.x + acc1.y));
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(q, static_cast<float>(a.H)), a.eps)));
    if (!valid) return;
    const float2 inv2 = make_float2(inv, inv);
    uint4* yrow = reinterpret_cast<uint4*>(static_cast<T*>(a.y) + row * a.H);
#pragma unroll 2
    for (int j = 0; j < KPL; ++j) {
        const uint32_t k = gl + G * j;
        float2 f[N2], o[N2];
        float g[P], b[P];
        Pk<T>::unpack(srow[k], f);
        load_params<P, G>(params, k, g);
        load_params<P, G>(params + a.param_stride, k, b);
#pragma unroll
        for (int i = 0; i < N2; ++i) {
            const float2 y = __fmul2_rn(__fadd2_rn(f[i], nmean), inv2);
            o[i] = __ffma2_rn(y, make_float2(g[2 * i], g[2 * i + 1]), make_float2(b[2 * i], b[2 * i + 1]));
        }
        __stcs(yrow + k, Pk<T>::pack(o));
    }
}

// RMSNorm + rotate-half RoPE over the whole row (rot == H, KPL = 2): lane gl owns pack gl of the
// first half and pack gl + G of the second half, which hold exactly each other's rotation
// partners, so the rotation needs no data from other lanes.  w0/w1: the lane's weights.
template <typename T, int G>
__device__ __forceinline__ void rms_rope_half_row(const NormArgs& a, const uint4* srow, const float2* w0,
                                                  const float2* w1, uint64_t row, uint32_t gl, bool valid) {
    constexpr int N2 = Pk<T>::N2, P = 2 * N2;
    float2 f0[N2], f1[N2];
    Pk<T>::unpack(srow[gl], f0);
    Pk<T>::unpack(srow[gl + G], f1);
    float2 acc0 = make_float2(0.f, 0.f), acc1 = acc0;
#pragma unroll
    for (int i = 0; i < N2; ++i) {
        acc0 = __ffma2_rn(f0[i], f0[i], acc0);
        acc1 = __ffma2_rn(f1[i], f1[i], acc1);
    }
    const float s = group_sum<G>((acc0.x + acc0.y) + (acc1.x + acc1.y));
    const float inv = rsqrtf(fmaf(s, a.inv_h, a.eps));
    if (!valid) return;
    const uint32_t pos = a.pos_of_row(static_cast<uint32_t>(row));
    const size_t t0 = static_cast<size_t>(pos) * (G * P) + gl * P;  // table row of H/2 entries
    float c[P], z[P];
    ldg_f32<P>(a.cos_t + t0, c);
    ldg_f32<P>(a.sin_t + t0, z);
    const float2 inv2 = make_float2(inv, inv);
    float2 o0[N2], o1[N2];
#pragma unroll
    for (int i = 0; i < N2; ++i) {
        const float2 y0 = __fmul2_rn(__fmul2_rn(f0[i], inv2), w0[i]);
        const float2 y1 = __fmul2_rn(__fmul2_rn(f1[i], inv2), w1[i]);
        const float2 c2 = make_float2(c[2 * i], c[2 * i + 1]), z2 = make_float2(z[2 * i], z[2 * i + 1]);
        o0[i] = __ffma2_rn(y0, c2, __fmul2_rn(make_float2(-y1.x, -y1.y), z2));  // y c - p s
        o1[i] = __ffma2_rn(y1, c2, __fmul2_rn(y0, z2));                         // y c + p s
    }
    uint4* yrow = reinterpret_cast<uint4*>(static_cast<T*>(a.y) + row * a.H);
    __stcs(yrow + gl, Pk<T>::pack(o0));
    __stcs(yrow + gl + G, Pk<T>::pack(o1));
}

// ---- named barriers of one consumer group (4 warps, 128 threads; ids 1..kGroups) ----
__device__ __forceinline__ void group_bar_sync(uint32_t id) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(kGroupWarps * 32) : "memory");
}
// Sums (a, b) over the group's 128 threads with one barrier (2 x kGroupWarps floats at `slot`).
__device__ __forceinline__ float2 group_reduce2(float a, float b, float* slot, uint32_t id, uint32_t gw, uint32_t lane) {
    a = group_sum<32>(a);
    b = group_sum<32>(b);
    if (lane == 0) {
        slot[gw] = a;
        slot[kGroupWarps + gw] = b;
    }
    group_bar_sync(id);
    float2 t = make_float2(0.f, 0.f);
#pragma unroll
    for (uint32_t w = 0; w < kGroupWarps; ++w) {
        t.x += slot[w];
        t.y += slot[kGroupWarps + w];
    }
    return t;
}

// Row-processing variants of the row-stream kernel.
enum RowMode : int { kGeneric = 0, kLnFast = 1, kRopeHalfFast = 2 };

template <typename T, NormKind KIND, int G, int MODE = kGeneric, int KPL = 1>
__global__ void __launch_bounds__(kThreads, 1) rowstream_kernel(NormArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    float* params = reinterpret_cast<float*>(smem);
    uint8_t* ring = smem + ((a.param_floats * 4 + 127) & ~127u);
    RingBars* bars = reinterpret_cast<RingBars*>(ring + a.stages * a.tile_bytes);
    volatile uint32_t* abort_flag = reinterpret_cast<uint32_t*>(bars + 1);
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const uint64_t num_tiles = (a.rows + a.tile_rows - 1) / a.tile_rows;
    const size_t row_bytes = static_cast<size_t>(a.H) * sizeof(T);

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < a.stages; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], kGroupWarps);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    // Stage the per-column parameters once per CTA, lane-transposed (see param_slot).
    {
        constexpr uint32_t P = elem<T>::kPack;
        for (uint32_t i = threadIdx.x; i < a.H; i += blockDim.x) {
            const uint32_t slot = param_slot<P, G>(i / P, (i % P) / 4) + i % 4;
            params[slot] = a.gamma[i];
            if (KIND == NormKind::kLayerNorm) params[a.param_stride + slot] = a.beta[i];
        }
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ================================ producer ================================
        if (lane == 0) {
            uint32_t stage = 0, phase = 0, pend_valid = 0, pend_phase = 0;
            bool ok = true;
            for (uint64_t t = blockIdx.x; t < num_tiles; t += gridDim.x) {
                if (!mbar_wait_bounded(&bars->empty[stage], phase ^ 1, abort_flag, &g_norm_error_word, 1u)) {
                    ok = false;
                    break;
                }
                const uint64_t r0 = t * a.tile_rows;
                const uint64_t nr = (a.rows - r0 < a.tile_rows) ? (a.rows - r0) : a.tile_rows;
                const uint32_t bytes = static_cast<uint32_t>(nr * row_bytes);
                mbar_arrive_expect_tx(&bars->full[stage], bytes);
                asm volatile(
                    "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                        smem_u32(ring + stage * a.tile_bytes)),
                    "l"(static_cast<const uint8_t*>(a.x) + r0 * row_bytes), "r"(bytes), "r"(smem_u32(&bars->full[stage]))
                    : "memory");
                pend_valid |= 1u << stage;
                pend_phase = (pend_phase & ~(1u << stage)) | (phase << stage);
                if (++stage == a.stages) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            if (!ok) {  // drain copies still in flight before the CTA's shared memory goes away
                volatile uint32_t never = 0;
                for (uint32_t s = 0; s < a.stages; ++s)
                    if (pend_valid & (1u << s))
                        mbar_wait_bounded(&bars->full[s], (pend_phase >> s) & 1u, &never, &g_norm_error_word, 4u,
                                          1000000000ull);
            }
        }
    } else {
        // ================================ consumers ================================
        constexpr uint32_t kRowsPerPass = 32 / G;
        const uint32_t sub = lane / G, gl = lane % G;
        const uint32_t grp = warp / kGroupWarps, gw = warp % kGroupWarps;
        // kRopeHalfFast: this lane's weights stay in registers for the whole kernel.
        constexpr int kN2 = Pk<T>::N2;
        float2 w0[kN2], w1[kN2];
        if constexpr (MODE == kRopeHalfFast) {
            float wf[2 * kN2];
            ldg_f32<2 * kN2>(a.gamma + gl * 2 * kN2, wf);
#pragma unroll
            for (int i = 0; i < kN2; ++i) w0[i] = make_float2(wf[2 * i], wf[2 * i + 1]);
            ldg_f32<2 * kN2>(a.gamma + (gl + G) * 2 * kN2, wf);
#pragma unroll
            for (int i = 0; i < kN2; ++i) w1[i] = make_float2(wf[2 * i], wf[2 * i + 1]);
        }
        for (uint64_t i = grp; grp < a.groups; i += a.groups) {
            const uint64_t t = blockIdx.x + i * gridDim.x;
            if (t >= num_tiles) break;
            const uint32_t stage = static_cast<uint32_t>(i % a.stages);
            const uint32_t phase = static_cast<uint32_t>((i / a.stages) & 1);
            bool ok = mbar_wait_bounded(&bars->full[stage], phase, abort_flag, &g_norm_error_word, 2u);
            if (!__all_sync(0xffffffffu, ok)) break;
            const uint64_t r0 = t * a.tile_rows;
            const uint32_t nr = static_cast<uint32_t>((a.rows - r0 < a.tile_rows) ? (a.rows - r0) : a.tile_rows);
            const uint8_t* tile = ring + stage * a.tile_bytes;
            for (uint32_t rb = gw * kRowsPerPass; rb < nr; rb += kGroupWarps * kRowsPerPass) {
                const uint32_t rr = rb + sub;
                const bool valid = rr < nr;
                const uint8_t* srow = tile + (valid ? rr : rb) * row_bytes;
                if constexpr (MODE == kLnFast)
                    ln_row_fast<T, G, KPL>(a, reinterpret_cast<const uint4*>(srow), params, r0 + rr, gl, valid);
                else if constexpr (MODE == kRopeHalfFast)
                    rms_rope_half_row<T, G>(a, reinterpret_cast<const uint4*>(srow), w0, w1, r0 + rr, gl, valid);
                else
                    process_row<T, KIND, G>(a, reinterpret_cast<const pack<T>*>(srow), params, r0 + rr, gl, valid);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->empty[stage]);
        }
    }
    __syncthreads();
}

// LayerNorm for long rows (H = 1024 * KPL 16-bit elements, or 512 * KPL fp32), direct form:
// no staging ring.  Each group of 128 threads owns whole rows (rows gg, gg + NG, ... for global
// group gg of NG); a thread keeps its KPL packs of the current row in registers and issues the
// streaming loads of its next row before working on the current one, so every group has two
// rows in flight.  Statistics as in ln_group_row (one pass over deviations from the row's first
// element, exact centred pass when that shift is far from the mean), combined across the group's
// four warps through shared memory and a named barrier; the reduction slots alternate by row
// parity so that a row's first write can never overwrite values of the previous row still being
// read.  No waits other than those barriers, which every thread of a group reaches the same
// number of times.
constexpr uint32_t kDirectGroups = 6;

template <typename T, int KPL>
__global__ void __launch_bounds__(kDirectGroups * kGroupWarps * 32, 1) ln_direct_kernel(NormArgs a) {
    constexpr int N2 = Pk<T>::N2, P = 2 * N2, GT = kGroupWarps * 32;
    extern __shared__ uint8_t smem_raw[];
    float* params = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    float* red_all = params + a.param_floats;  // kDirectGroups x 2 parities x 4 x kGroupWarps
    for (uint32_t i = threadIdx.x; i < a.H; i += blockDim.x) {
        const uint32_t slot = param_slot<P, GT>(i / P, (i % P) / 4) + i % 4;
        params[slot] = a.gamma[i];
        params[a.param_stride + slot] = a.beta[i];
    }
    __syncthreads();
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const uint32_t grp = warp / kGroupWarps, gw = warp % kGroupWarps, tid = gw * 32 + lane;
    const uint32_t bar_id = 1 + grp;
    float* red_grp = red_all + grp * 2 * 4 * kGroupWarps;
    const uint64_t NG = static_cast<uint64_t>(gridDim.x) * kDirectGroups;
    const uint4* x = static_cast<const uint4*>(a.x);
    const uint64_t row_packs = a.H / P;

    const uint16_t* x16 = static_cast<const uint16_t*>(a.x);  // first element of a row (K), any T
    auto first_elem = [&](uint64_t r) -> float {
        if constexpr (sizeof(T) == 4) return __uint_as_float(__ldg(reinterpret_cast<const uint32_t*>(a.x) + r * a.H));
        else {
            const uint16_t bits = __ldg(x16 + r * a.H);
            return elem<T>::to_f(*reinterpret_cast<const T*>(&bits));
        }
    };
    uint64_t row = static_cast<uint64_t>(blockIdx.x) * kDirectGroups + grp;
    uint4 cur[KPL];
    float Kr = 0.f;
    if (row < a.rows) {
#pragma unroll
        for (int j = 0; j < KPL; ++j) cur[j] = __ldcs(x + row * row_packs + tid + GT * j);
        Kr = first_elem(row);
    }
    for (uint32_t it = 0; row < a.rows; ++it, row += NG) {
        // prefetch the group's next row (and its first element)
        uint4 nxt[KPL];
        float Kn = 0.f;
        const uint64_t nrow = row + NG;
        if (nrow < a.rows) {
#pragma unroll
            for (int j = 0; j < KPL; ++j) nxt[j] = __ldcs(x + nrow * row_packs + tid + GT * j);
            Kn = first_elem(nrow);
        }
        float* red = red_grp + (it & 1) * 4 * kGroupWarps;
        const float2 nk = make_float2(-Kr, -Kr);
        float2 s1 = make_float2(0.f, 0.f), s2 = s1;
#pragma unroll
        for (int j = 0; j < KPL; ++j) {
            float2 f[N2];
            Pk<T>::unpack(cur[j], f);
#pragma unroll
            for (int i = 0; i < N2; ++i) {
                const float2 d = __fadd2_rn(f[i], nk);
                s1 = __fadd2_rn(s1, d);
                s2 = __ffma2_rn(d, d, s2);
            }
        }
        const float2 tot = group_reduce2(s1.x + s1.y, s2.x + s2.y, red, bar_id, gw, lane);
        const float dm = __fdiv_rn(tot.x, static_cast<float>(a.H));  // mean - K
        const float mean = __fadd_rn(Kr, dm);
        float var = fmaxf(__fsub_rn(__fdiv_rn(tot.y, static_cast<float>(a.H)), __fmul_rn(dm, dm)), 0.f);
        const float2 nmean = make_float2(-mean, -mean);
        if (dm * dm > 16.f * var) {  // group-uniform: exact centred pass
            float2 q = make_float2(0.f, 0.f);
#pragma unroll
            for (int j = 0; j < KPL; ++j) {
                float2 f[N2];
                Pk<T>::unpack(cur[j], f);
#pragma unroll
                for (int i = 0; i < N2; ++i) {
                    const float2 d = __fadd2_rn(f[i], nmean);
                    q = __ffma2_rn(d, d, q);
                }
            }
            var = __fdiv_rn(group_reduce2(q.x + q.y, 0.f, red + 2 * kGroupWarps, bar_id, gw, lane).x,
                            static_cast<float>(a.H));
        }
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, a.eps)));
        const float2 inv2 = make_float2(inv, inv);
        uint4* yrow = reinterpret_cast<uint4*>(static_cast<T*>(a.y) + row * a.H);
#pragma unroll
        for (int j = 0; j < KPL; ++j) {
            const uint32_t k = tid + GT * j;
            float2 f[N2], o[N2];
            float g[P], b[P];
            Pk<T>::unpack(cur[j], f);
            load_params<P, GT>(params, k, g);
            load_params<P, GT>(params + a.param_stride, k, b);
#pragma unroll
            for (int i = 0; i < N2; ++i) {
                const float2 y = __fmul2_rn(__fadd2_rn(f[i], nmean), inv2);
                o[i] = __ffma2_rn(y, make_float2(g[2 * i], g[2 * i + 1]), make_float2(b[2 * i], b[2 * i + 1]));
            }
            __stcs(yrow + k, Pk<T>::pack(o));
        }
#pragma unroll
        for (int j = 0; j < KPL; ++j) cur[j] = nxt[j];
        Kr = Kn;
    }
}

template <typename T, int KPL>
int launch_ln_direct(NormArgs a, cudaStream_t s) {
    constexpr uint32_t P = elem<T>::kPack, GT = kGroupWarps * 32;
    a.param_stride = a.H / P / GT * GT * P;  // = H: packs are a multiple of GT
    a.param_floats = 2 * a.param_stride;
    const size_t smem = 128 + static_cast<size_t>(a.param_floats) * 4 + kDirectGroups * 2 * 4 * kGroupWarps * 4;
    if (int rc = set_max_dynamic_smem(reinterpret_cast<const void*>(ln_direct_kernel<T, KPL>), smem, "ln_direct_kernel"))
        return rc;
    const uint64_t groups_needed = (static_cast<uint64_t>(a.rows) + 1) / 2;  // two rows per group at least
    uint64_t grid = (groups_needed + kDirectGroups - 1) / kDirectGroups;
    if (grid > static_cast<uint64_t>(sm_count())) grid = sm_count();
    if (grid == 0) grid = 1;
    // Rows go round-robin over grid * kDirectGroups groups, so the launch lasts ceil(rows / groups)
    // row rounds.  Among grids of at least 85 % of the SMs, take the one whose rounds leave the
    // fewest row slots idle (16384 rows: 144 CTAs, 0.2 % idle slots instead of 3 % at 148; measured
    // +0.5 points of HBM bandwidth, since the row prefetch already overlaps consecutive rounds).
    {
        const uint64_t rows = a.rows, g_hi = grid, g_lo = (g_hi * 85 + 99) / 100;
        uint64_t best = g_hi, best_slots = ((rows + g_hi * kDirectGroups - 1) / (g_hi * kDirectGroups)) * g_hi * kDirectGroups;
        for (uint64_t g = g_hi; g >= g_lo && g >= 1; --g) {
            const uint64_t slots = ((rows + g * kDirectGroups - 1) / (g * kDirectGroups)) * g * kDirectGroups;
            if (slots < best_slots) {
                best_slots = slots;
                best = g;
            }
        }
        grid = best;
    }
    ln_direct_kernel<T, KPL><<<static_cast<unsigned>(grid), kDirectGroups * GT, smem, s>>>(a);
    return check_launch("layer_norm");
}

// Scalar fallback (unaligned buffers or rows that are not a multiple of 16 bytes): one block per
// row, three passes over the row staged in shared memory.
template <typename T, NormKind KIND>
__global__ void __launch_bounds__(256) rownorm_scalar_kernel(NormArgs a) {
    __shared__ float red[8];
    extern __shared__ float row_buf[];  // H floats
    const T* x = static_cast<const T*>(a.x);
    T* y = static_cast<T*>(a.y);
    for (uint64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
        const T* xr = x + row * a.H;
        const float K = (KIND == NormKind::kLayerNorm) ? elem<T>::to_f(xr[0]) : 0.f;  // LayerNorm shift
        float s = 0.f;
        for (uint32_t d = threadIdx.x; d < a.H; d += blockDim.x) {
            float v = elem<T>::to_f(xr[d]);
            row_buf[d] = v;
            s = (KIND == NormKind::kLayerNorm) ? __fadd_rn(s, __fsub_rn(v, K)) : __fadd_rn(s, __fmul_rn(v, v));
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
        float mul, shift = 0.f;
        if (KIND == NormKind::kLayerNorm) {
            float mean = __fadd_rn(K, __fdiv_rn(s, static_cast<float>(a.H)));
            float q = 0.f;
            for (uint32_t d = threadIdx.x; d < a.H; d += blockDim.x) {
                float dd = __fsub_rn(row_buf[d], mean);
                q = __fadd_rn(q, __fmul_rn(dd, dd));
            }
            q = block_sum(q);
            mul = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(q, static_cast<float>(a.H)), a.eps)));
            shift = mean;
        } else {
            mul = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, static_cast<float>(a.H)), a.eps)));
        }
        for (uint32_t d = threadIdx.x; d < a.H; d += blockDim.x) {
            float v = row_buf[d];
            if (KIND == NormKind::kLayerNorm)
                v = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v, shift), mul), a.gamma[d]), a.beta[d]);
            else
                v = __fmul_rn(__fmul_rn(v, mul), a.gamma[d]);
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

uint32_t read_error_word(const char** name) {
    *name = "layer_norm/rms_norm_rope_fused row stream";
    uint32_t word = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&word, g_norm_error_word, sizeof(word)) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (word) cudaMemcpyToSymbol(g_norm_error_word, &zero, sizeof(zero));
    return word;
}

template <typename T, NormKind KIND, int G, int MODE = kGeneric, int KPL = 1>
int launch_rowstream(NormArgs a, cudaStream_t s) {
    static std::once_flag reg_once;
    std::call_once(reg_once, [] { register_error_word(read_error_word); });
    constexpr uint32_t P = elem<T>::kPack;
    const uint32_t packs = a.H / P;
    a.param_stride = (packs + G - 1) / G * G * P;
    a.param_floats = (KIND == NormKind::kLayerNorm ? 2 : 1) * a.param_stride;
    if (a.param_floats * 4ull > 64 * 1024) return fail(HC_ERR_UNSUPPORTED, "row of %u elements too long", a.H);
    a.vec_rope = (KIND == NormKind::kRmsRope) && a.rot % P == 0 && (a.rot / 2) % P == 0 &&
                 (a.rot / 2) % 4 == 0 && aligned16(a.cos_t) && aligned16(a.sin_t);
    a.xor_partner = a.vec_rope && a.style == 1 && a.rot == a.H && packs == G;
    a.div_heads.init(a.heads);
    a.div_S.init(a.S);
    const uint32_t row_bytes = a.H * static_cast<uint32_t>(sizeof(T));
    const uint32_t rows_per_pass = kGroupWarps * (32 / G);  // rows one consumer group takes at once
    const uint32_t param_bytes = ((a.param_floats * 4 + 127) & ~127u);
    // Tile: whole passes of a consumer group, up to 16 KB when rows allow.
    uint32_t passes = 1;
    while (passes < 64 && rows_per_pass * (passes * 2) * row_bytes <= 16 * 1024) passes *= 2;
    a.tile_rows = rows_per_pass * passes;
    if (static_cast<uint64_t>(a.tile_rows) * row_bytes > 64 * 1024) {
        a.tile_rows = (64 * 1024) / row_bytes;
        if (a.tile_rows == 0) a.tile_rows = 1;
    }
    a.tile_bytes = a.tile_rows * row_bytes;
    const uint32_t bar_bytes = sizeof(RingBars) + 16;
    uint32_t avail = kSmemBudget - param_bytes - bar_bytes - 128;
    a.stages = avail / a.tile_bytes;
    if (a.stages > kMaxStages) a.stages = kMaxStages;
    if (a.stages < 2) {
        a.tile_rows = 1;
        a.tile_bytes = row_bytes;
        a.stages = avail / a.tile_bytes;
        if (a.stages > kMaxStages) a.stages = kMaxStages;
        if (a.stages < 2) return fail(HC_ERR_UNSUPPORTED, "row of %u bytes too long for the row-stream kernel", row_bytes);
    }
    a.groups = a.stages - 1 < kGroups ? a.stages - 1 : kGroups;  // keep one stage filling
    const size_t smem = 128 + param_bytes + static_cast<size_t>(a.stages) * a.tile_bytes + bar_bytes;
    if (int rc = set_max_dynamic_smem(reinterpret_cast<const void*>(rowstream_kernel<T, KIND, G, MODE, KPL>),
                                      kSmemBudget + 1024, "rowstream_kernel"))
        return rc;
    const uint64_t tiles = (a.rows + a.tile_rows - 1) / a.tile_rows;
    const uint64_t grid = tiles < static_cast<uint64_t>(sm_count()) ? tiles : static_cast<uint64_t>(sm_count());
    rowstream_kernel<T, KIND, G, MODE, KPL><<<static_cast<unsigned>(grid), kThreads, smem, s>>>(a);
    return check_launch(KIND == NormKind::kLayerNorm ? "layer_norm" : "rms_norm_rope_fused");
}

template <typename T, NormKind KIND>
int launch_rownorm(NormArgs a, void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    constexpr uint32_t P = elem<T>::kPack;
    a.param_floats = (KIND == NormKind::kLayerNorm ? 2 : 1) * a.H;
    const uint32_t packs = a.H / P;
    const bool stream_ok = (a.H % P == 0) && aligned16(a.x) && aligned16(a.y) &&
                           a.param_floats * 4ull <= 64 * 1024;
    if (stream_ok) {
        if constexpr (KIND == NormKind::kLayerNorm) {
            switch (packs) {  // long rows of 128 * KPL packs: one 128-thread group per row, direct loads
                case 128: return launch_ln_direct<T, 1>(a, s);
                case 256: return launch_ln_direct<T, 2>(a, s);
                case 512: return launch_ln_direct<T, 4>(a, s);
                default: break;
            }
            switch (packs) {  // rows of exactly 32 * KPL packs: the unrolled LayerNorm
                case 64: return launch_rowstream<T, KIND, 32, kLnFast, 2>(a, s);
                case 128: return launch_rowstream<T, KIND, 32, kLnFast, 4>(a, s);
                case 256: return launch_rowstream<T, KIND, 32, kLnFast, 8>(a, s);
                case 512: return launch_rowstream<T, KIND, 32, kLnFast, 16>(a, s);
                default: break;
            }
        } else {
            // rotate-half over the whole row with 16-byte-aligned tables: lane-local partners
            // (weights and tables are read as 16-byte vectors: all three must be 16-byte aligned)
            const bool half_local = a.style == 1 && a.rot == a.H && aligned16(a.cos_t) && aligned16(a.sin_t) &&
                                    aligned16(a.gamma) && (a.H / 2) % 4 == 0;
            if (half_local && packs == 16) return launch_rowstream<T, KIND, 8, kRopeHalfFast, 2>(a, s);
            if (half_local && packs == 32) return launch_rowstream<T, KIND, 16, kRopeHalfFast, 2>(a, s);
        }
        if (packs >= 32) return launch_rowstream<T, KIND, 32>(a, s);
        if (packs >= 16) return launch_rowstream<T, KIND, 16>(a, s);
        return launch_rowstream<T, KIND, 8>(a, s);
    }
    size_t smem = static_cast<size_t>(a.H) * sizeof(float);
    if (smem > 200 * 1024) return fail(HC_ERR_UNSUPPORTED, "row length %u too long for the scalar row kernel", a.H);
    if (smem > 48 * 1024) {
        if (int rc = set_max_dynamic_smem(reinterpret_cast<const void*>(rownorm_scalar_kernel<T, KIND>), smem,
                                          "rownorm_scalar_kernel"))
            return rc;
    }
    const uint64_t cap =
        static_cast<uint64_t>(resident_blocks(reinterpret_cast<const void*>(rownorm_scalar_kernel<T, KIND>), 256, smem));
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
    a.inv_h = 1.0f / static_cast<float>(t->H);
    return dispatch_rownorm<NormKind::kRmsRope>(dtype, a, stream, "rms_norm_rope_fused");
}
