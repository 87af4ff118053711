// Elementwise ladder operators: elementwise_add, axpy_scalar_affine, broadcast_binary,
// activation_gelu_silu.  All are HBM-bound streams: 16-byte packs, grid-stride loops sized to
// the SM count, no tensor cores.
//
// Arithmetic follows the reference goldens operation by operation, with explicitly rounded
// fp32 intrinsics so the compiler cannot contract a*b+c into one FMA (the goldens are compiled
// for x86-64 without FMA, so each product and sum is rounded separately):
//   elementwise_add      ops/elementwise_add/golden/elementwise_add_golden.cpp:12-14
//   axpy_scalar_affine   ops/axpy_scalar_affine/golden/axpy_scalar_affine_golden.cpp:13-15
//   broadcast_binary     ops/broadcast_binary/golden/broadcast_binary_golden.cpp:28-40
//   activation_gelu_silu ops/activation_gelu_silu/golden/activation_gelu_silu_golden.cpp:16-49
//                        (fp32; bf16/fp16 use the sigmoid form of FastActOp, see there)
#include <cuda_runtime.h>

#include "hc_device.cuh"
#include "hc_internal.h"

namespace hc {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

// Grid of a grid-stride launch: one block per kThreads * kUnroll work items, at most as many
// blocks as are resident at once.
template <typename K>
int grid_for(K kernel, size_t work_items) {
    size_t blocks = (work_items + kThreads * kUnroll - 1) / (kThreads * kUnroll);
    const size_t cap = static_cast<size_t>(resident_blocks(reinterpret_cast<const void*>(kernel), kThreads, 0));
    if (blocks > cap) blocks = cap;
    if (blocks == 0) blocks = 1;
    return static_cast<int>(blocks);
}

// Ops with apply2 (a float2 pair at a time) take the paired path of map2_vec_kernel.
template <typename Op, typename = void>
struct has_apply2 {
    static constexpr bool value = false;
};
template <typename Op>
struct has_apply2<Op, decltype(void(&Op::apply2))> {
    static constexpr bool value = true;
};

// ---------------------------------------------------------------------------------------
// Generic unary/binary maps.  Op::apply(float a, float b) -> float.
// ---------------------------------------------------------------------------------------
template <typename T, typename Op>
__global__ void __launch_bounds__(kThreads) map2_vec_kernel(const T* __restrict__ a, const T* __restrict__ b,
                                                            T* __restrict__ out, size_t n, Op op) {
    constexpr int P = elem<T>::kPack;
    const size_t packs = n / P;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    const pack<T>* pa = reinterpret_cast<const pack<T>*>(a);
    const pack<T>* pb = reinterpret_cast<const pack<T>*>(b);
    pack<T>* po = reinterpret_cast<pack<T>*>(out);
    size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    for (; i + (kUnroll - 1) * stride < packs; i += kUnroll * stride) {
        pack<T> va[kUnroll], vb[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            va[u] = ld_stream(pa + i + u * stride);
            if (Op::kBinary) vb[u] = ld_stream(pb + i + u * stride);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            pack<T> r;
            if constexpr (has_apply2<Op>::value) {
#pragma unroll
                for (int e = 0; e < P; e += 2) {
                    const float2 f = op.apply2(make_float2(elem<T>::to_f(va[u].v[e]), elem<T>::to_f(va[u].v[e + 1])));
                    r.v[e] = elem<T>::from_f(f.x);
                    r.v[e + 1] = elem<T>::from_f(f.y);
                }
            } else {
#pragma unroll
                for (int e = 0; e < P; ++e)
                    r.v[e] = elem<T>::from_f(
                        op.apply(elem<T>::to_f(va[u].v[e]), Op::kBinary ? elem<T>::to_f(vb[u].v[e]) : 0.f));
            }
            st_stream(po + i + u * stride, r);
        }
    }
    for (; i < packs; i += stride) {
        pack<T> va = ld_stream(pa + i);
        pack<T> vb;
        if (Op::kBinary) vb = ld_stream(pb + i);
        pack<T> r;
#pragma unroll
        for (int e = 0; e < P; ++e)
            r.v[e] = elem<T>::from_f(op.apply(elem<T>::to_f(va.v[e]), Op::kBinary ? elem<T>::to_f(vb.v[e]) : 0.f));
        st_stream(po + i, r);
    }
    // Tail elements that do not fill a pack.
    const size_t tail0 = packs * P;
    const size_t gtid = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (gtid < n - tail0) {
        size_t j = tail0 + gtid;
        out[j] = elem<T>::from_f(op.apply(elem<T>::to_f(a[j]), Op::kBinary ? elem<T>::to_f(b[j]) : 0.f));
    }
}

// Scalar variant for buffers that are not 16-byte aligned.
template <typename T, typename Op>
__global__ void __launch_bounds__(kThreads) map2_scalar_kernel(const T* __restrict__ a, const T* __restrict__ b,
                                                               T* __restrict__ out, size_t n, Op op) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t j = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; j < n; j += stride)
        out[j] = elem<T>::from_f(op.apply(elem<T>::to_f(a[j]), Op::kBinary ? elem<T>::to_f(b[j]) : 0.f));
}

struct AddOp {
    static constexpr bool kBinary = true;
    // One fp32 add, then one rounding to the storage type.  For fp16/bf16 inputs the fp32 sum
    // is exact-or-correctly-rounded with p=24 >= 2p'+2, so the result equals the correctly
    // rounded 16-bit addition (what __hadd2 computes).
    __device__ float apply(float x, float y) const { return __fadd_rn(x, y); }
};

struct AxpyOp {
    static constexpr bool kBinary = false;
    float alpha, beta;
    __device__ float apply(float x, float) const { return __fadd_rn(__fmul_rn(alpha, x), beta); }
};

struct ActOp {
    static constexpr bool kBinary = false;
    uint32_t act;  // 0 = GELU (tanh form), 1 = SiLU
    __device__ float apply(float v, float) const {
        if (act == 0) {
            const float kSqrt2OverPi = 0.7978845608f;
            const float kGeluCoeff = 0.044715f;
            float x3 = __fmul_rn(__fmul_rn(v, v), v);
            float inner = __fmul_rn(kSqrt2OverPi, __fadd_rn(v, __fmul_rn(kGeluCoeff, x3)));
            float t = tanhf(inner);
            return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, t));
        }
        if (v >= 0.0f) {
            float e = expf(-v);
            return __fdiv_rn(v, __fadd_rn(1.0f, e));
        }
        float e = expf(v);
        return __fdiv_rn(__fmul_rn(v, e), __fadd_rn(1.0f, e));
    }
};

// 16-bit outputs: the same functions through the logistic sigmoid, which needs one exponential
// and one reciprocal instead of tanhf / expf / IEEE division:
//   GELU_tanh(x) = 0.5 x (1 + tanh u) = x * sigmoid(2u),  u = sqrt(2/pi) (x + 0.044715 x^3);
//   SiLU(x) = x * sigmoid(x);  sigmoid(z) = 1 / (1 + 2^(-z log2 e)).
// With the constants folded into the base-2 exponent, both are x / (1 + 2^y), y = -x (a + b x^2):
// GELU a = 2 sqrt(2/pi) log2 e, b = 0.044715 a; SiLU a = log2 e, b = 0.  Relative error ~1e-6, far
// below the rounding of the bf16/fp16 result (2^-9 / 2^-12); the fp32 path (ActOp) keeps the
// golden's operation order.  y is clamped to 126, so 1 + 2^y stays finite: for x -> -inf the
// result is x * 2^-126-ish, i.e. 0 after rounding to 16 bits, as the golden gives.
__device__ __forceinline__ float ex2_ftz(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float rcp_ftz(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

struct FastActOp {
    static constexpr bool kBinary = false;
    float a, b;  // y = -x (a + b x^2)
    __host__ static FastActOp make(uint32_t act) {
        const double log2e = 1.4426950408889634;
        const double k = 2.0 * 0.7978845608028654 * log2e;  // 2 sqrt(2/pi) log2 e
        return act == 0 ? FastActOp{static_cast<float>(k), static_cast<float>(0.044715 * k)}
                        : FastActOp{static_cast<float>(log2e), 0.f};
    }
    __device__ float2 apply2(float2 x) const {
        const float2 w = __ffma2_rn(make_float2(-b, -b), __fmul2_rn(x, x), make_float2(-a, -a));
        const float2 y = __fmul2_rn(x, w);
        float2 d = make_float2(ex2_ftz(fminf(y.x, 126.f)), ex2_ftz(fminf(y.y, 126.f)));
        d = __fadd2_rn(d, make_float2(1.f, 1.f));
        // MUFU rcp: measured faster here than three Newton steps on the FMA pipe
        return __fmul2_rn(x, make_float2(rcp_ftz(d.x), rcp_ftz(d.y)));
    }
    __device__ float apply(float v, float) const { return apply2(make_float2(v, v)).x; }
};

template <typename T, typename Op>
int launch_map(const void* a, const void* b, void* out, size_t n, Op op, void* stream, const char* name) {
    if (n == 0) return ok();
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const T* ta = static_cast<const T*>(a);
    const T* tb = static_cast<const T*>(b);
    T* to = static_cast<T*>(out);
    bool vec = aligned16(a) && aligned16(out) && (!Op::kBinary || aligned16(b));
    if (vec) {
        size_t packs = n / elem<T>::kPack;
        map2_vec_kernel<T, Op><<<grid_for(map2_vec_kernel<T, Op>, packs > 0 ? packs : 1), kThreads, 0, s>>>(ta, tb, to, n, op);
    } else {
        map2_scalar_kernel<T, Op><<<grid_for(map2_scalar_kernel<T, Op>, n), kThreads, 0, s>>>(ta, tb, to, n, op);
    }
    return check_launch(name);
}

template <typename Op>
int dispatch_map(int dtype, const void* a, const void* b, void* out, size_t n, Op op, void* stream, const char* name) {
    switch (dtype) {
        case HC_DTYPE_F32: return launch_map<float, Op>(a, b, out, n, op, stream, name);
        case HC_DTYPE_F16: return launch_map<f16_t, Op>(a, b, out, n, op, stream, name);
        case HC_DTYPE_BF16: return launch_map<bf16_t, Op>(a, b, out, n, op, stream, name);
        default: return fail(HC_ERR_UNSUPPORTED, "%s: dtype %d not supported (F32, F16, BF16)", name, dtype);
    }
}

// ---------------------------------------------------------------------------------------
// broadcast_binary: z = x * y[yb, c] + bias[c]
// ---------------------------------------------------------------------------------------
// One pack never straddles two (b, c) planes (hw % P == 0).  Pack i lies in plane i / (hw / P);
// the plane splits into (b, c) = (plane / C, plane % C), both by multiply-shift division (the
// launcher takes this kernel only when the pack count fits 32 bits).
template <typename T>
__global__ void __launch_bounds__(kThreads) broadcast_vec_kernel(const T* __restrict__ x, const T* __restrict__ y,
                                                                 const T* __restrict__ bias, T* __restrict__ z,
                                                                 FastDiv plane_packs, FastDiv cdiv, bool y_per_batch,
                                                                 uint32_t packs) {
    constexpr int P = elem<T>::kPack;
    const uint32_t stride = gridDim.x * blockDim.x;
    const pack<T>* px = reinterpret_cast<const pack<T>*>(x);
    pack<T>* pz = reinterpret_cast<pack<T>*>(z);
    uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    for (; static_cast<uint64_t>(i) + (kUnroll - 1) * static_cast<uint64_t>(stride) < packs; i += kUnroll * stride) {
        pack<T> v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) v[u] = ld_stream(px + i + u * stride);
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const uint32_t plane = plane_packs.div(i + u * stride);
            const uint32_t b = cdiv.div(plane), c = plane - b * cdiv.d;
            const float yv = elem<T>::to_f(y[(y_per_batch ? b * cdiv.d : 0) + c]);
            const float bv = elem<T>::to_f(bias[c]);
            pack<T> r;
#pragma unroll
            for (int e = 0; e < P; ++e) r.v[e] = elem<T>::from_f(__fadd_rn(__fmul_rn(elem<T>::to_f(v[u].v[e]), yv), bv));
            st_stream(pz + i + u * stride, r);
        }
    }
    for (; i < packs; i += stride) {
        const pack<T> v = ld_stream(px + i);
        const uint32_t plane = plane_packs.div(i);
        const uint32_t b = cdiv.div(plane), c = plane - b * cdiv.d;
        const float yv = elem<T>::to_f(y[(y_per_batch ? b * cdiv.d : 0) + c]);
        const float bv = elem<T>::to_f(bias[c]);
        pack<T> r;
#pragma unroll
        for (int e = 0; e < P; ++e) r.v[e] = elem<T>::from_f(__fadd_rn(__fmul_rn(elem<T>::to_f(v.v[e]), yv), bv));
        st_stream(pz + i, r);
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) broadcast_scalar_kernel(const T* __restrict__ x, const T* __restrict__ y,
                                                                    const T* __restrict__ bias, T* __restrict__ z,
                                                                    uint32_t C, size_t hw, size_t chw, bool y_per_batch,
                                                                    size_t n) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t j = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; j < n; j += stride) {
        size_t b = j / chw;
        uint32_t c = static_cast<uint32_t>((j / hw) % C);
        float yv = elem<T>::to_f(y[(y_per_batch ? b * C : 0) + c]);
        float bv = elem<T>::to_f(bias[c]);
        z[j] = elem<T>::from_f(__fadd_rn(__fmul_rn(elem<T>::to_f(x[j]), yv), bv));
    }
}

template <typename T>
int launch_broadcast(const void* x, const void* y, const void* bias, void* z, const broadcast_binary_tiling_data* t,
                     void* stream) {
    size_t hw = static_cast<size_t>(t->H) * t->W;
    size_t chw = hw * t->C;
    size_t n = chw * t->B;
    bool per_batch = (t->y_batch == t->B) && t->B != 1;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const T* tx = static_cast<const T*>(x);
    const T* ty = static_cast<const T*>(y);
    const T* tb = static_cast<const T*>(bias);
    T* tz = static_cast<T*>(z);
    const size_t packs = n / elem<T>::kPack;
    if (aligned16(x) && aligned16(z) && hw % elem<T>::kPack == 0 && packs < (1ull << 32) - kThreads * kUnroll * 8ull * 1024) {
        FastDiv plane_packs, cdiv;
        plane_packs.init(static_cast<uint32_t>(hw / elem<T>::kPack));
        cdiv.init(t->C);
        broadcast_vec_kernel<T><<<grid_for(broadcast_vec_kernel<T>, packs), kThreads, 0, s>>>(tx, ty, tb, tz, plane_packs, cdiv, per_batch,
                                                                     static_cast<uint32_t>(packs));
    } else {
        broadcast_scalar_kernel<T><<<grid_for(broadcast_scalar_kernel<T>, n), kThreads, 0, s>>>(tx, ty, tb, tz, t->C, hw, chw, per_batch, n);
    }
    return check_launch("broadcast_binary");
}

}  // namespace
}  // namespace hc

using namespace hc;

extern "C" int hc_elementwise_add_launch(const void* x, const void* y, void* z, const elementwise_add_tiling_data* t,
                                         int dtype, void* stream) {
    if (!t) return fail(HC_ERR_INVALID, "elementwise_add: null tiling");
    if (t->totalLength && (!x || !y || !z)) return fail(HC_ERR_INVALID, "elementwise_add: null pointer");
    if (fault_hit("launch")) return fail(HC_ERR_INJECTED, "elementwise_add: injected launch failure");
    return dispatch_map(dtype, x, y, z, t->totalLength, AddOp{}, stream, "elementwise_add");
}

extern "C" int hc_axpy_scalar_affine_launch(const void* x, void* y, const axpy_scalar_affine_tiling_data* t, float alpha,
                                            float beta, int dtype, void* stream) {
    if (!t) return fail(HC_ERR_INVALID, "axpy_scalar_affine: null tiling");
    if (t->totalLength && (!x || !y)) return fail(HC_ERR_INVALID, "axpy_scalar_affine: null pointer");
    if (fault_hit("launch")) return fail(HC_ERR_INJECTED, "axpy_scalar_affine: injected launch failure");
    return dispatch_map(dtype, x, nullptr, y, t->totalLength, AxpyOp{alpha, beta}, stream, "axpy_scalar_affine");
}

extern "C" int hc_activation_gelu_silu_launch(const void* x, void* y, const activation_gelu_silu_tiling_data* t,
                                              int dtype, void* stream) {
    if (!t) return fail(HC_ERR_INVALID, "activation_gelu_silu: null tiling");
    if (t->actType > 1) return fail(HC_ERR_INVALID, "activation_gelu_silu: actType %u (0 = GELU, 1 = SiLU)", t->actType);
    if (t->totalLength && (!x || !y)) return fail(HC_ERR_INVALID, "activation_gelu_silu: null pointer");
    if (fault_hit("launch")) return fail(HC_ERR_INJECTED, "activation_gelu_silu: injected launch failure");
    if (dtype == HC_DTYPE_F32)
        return dispatch_map(dtype, x, nullptr, y, t->totalLength, ActOp{t->actType}, stream, "activation_gelu_silu");
    return dispatch_map(dtype, x, nullptr, y, t->totalLength, FastActOp::make(t->actType), stream, "activation_gelu_silu");
}

extern "C" int hc_broadcast_binary_launch(const void* x, const void* y, const void* bias, void* z,
                                          const broadcast_binary_tiling_data* t, int dtype, void* stream) {
    if (!t) return fail(HC_ERR_INVALID, "broadcast_binary: null tiling");
    // Same argument checks as ops/broadcast_binary/golden/broadcast_binary_golden.cpp:14-22.
    if (!x || !y || !bias || !z) return fail(HC_ERR_INVALID, "broadcast_binary: null pointer");
    if (t->B == 0 || t->C == 0 || t->H == 0 || t->W == 0) return fail(HC_ERR_INVALID, "broadcast_binary: invalid dimensions");
    if (t->y_batch != 1 && t->y_batch != t->B) return fail(HC_ERR_INVALID, "broadcast_binary: y_batch must be 1 or B");
    if (fault_hit("launch")) return fail(HC_ERR_INJECTED, "broadcast_binary: injected launch failure");
    switch (dtype) {
        case HC_DTYPE_F32: return launch_broadcast<float>(x, y, bias, z, t, stream);
        case HC_DTYPE_F16: return launch_broadcast<f16_t>(x, y, bias, z, t, stream);
        case HC_DTYPE_BF16: return launch_broadcast<bf16_t>(x, y, bias, z, t, stream);
        default: return fail(HC_ERR_UNSUPPORTED, "broadcast_binary: dtype %d not supported", dtype);
    }
}
