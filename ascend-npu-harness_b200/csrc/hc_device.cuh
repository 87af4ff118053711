// Device-side helpers shared by the bandwidth-bound operator kernels: element conversions,
// 16-byte packs, streaming loads/stores and warp reductions.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

namespace hc {

// Storage types.  16-bit floats travel as raw bits so one template handles both formats.
struct bf16_t { uint16_t bits; };
struct f16_t { uint16_t bits; };

template <typename T> struct elem;
template <> struct elem<float> {
    static constexpr int kPack = 4;
    __device__ static float to_f(float v) { return v; }
    __device__ static float from_f(float v) { return v; }
};
template <> struct elem<bf16_t> {
    static constexpr int kPack = 8;
    __device__ static float to_f(bf16_t v) { return __uint_as_float(static_cast<uint32_t>(v.bits) << 16); }
    __device__ static bf16_t from_f(float v) {
        __nv_bfloat16 h = __float2bfloat16_rn(v);
        return bf16_t{*reinterpret_cast<uint16_t*>(&h)};
    }
};
template <> struct elem<f16_t> {
    static constexpr int kPack = 8;
    __device__ static float to_f(f16_t v) { return __half2float(*reinterpret_cast<const __half*>(&v.bits)); }
    __device__ static f16_t from_f(float v) {
        __half h = __float2half_rn(v);
        return f16_t{*reinterpret_cast<uint16_t*>(&h)};
    }
};

// 16-byte pack of elements.
template <typename T>
struct alignas(16) pack {
    T v[elem<T>::kPack];
};

// Loads that bypass L1 allocation (streamed once) and evict-first stores.
template <typename T>
__device__ __forceinline__ pack<T> ld_stream(const pack<T>* p) {
    uint4 r = __ldcs(reinterpret_cast<const uint4*>(p));
    return *reinterpret_cast<pack<T>*>(&r);
}
template <typename T>
__device__ __forceinline__ pack<T> ld_cached(const pack<T>* p) {
    uint4 r = __ldg(reinterpret_cast<const uint4*>(p));
    return *reinterpret_cast<pack<T>*>(&r);
}
template <typename T>
__device__ __forceinline__ void st_stream(pack<T>* p, const pack<T>& v) {
    __stcs(reinterpret_cast<uint4*>(p), *reinterpret_cast<const uint4*>(&v));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__host__ __device__ __forceinline__ bool aligned16(const void* p) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// Converts P floats to one 16-byte pack (16-bit types two at a time).
template <typename T>
__device__ __forceinline__ pack<T> pack_from_f(const float* f) {
    pack<T> o;
    if constexpr (sizeof(T) == 2) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if constexpr (std::is_same<T, bf16_t>::value) {
                __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
                w[i] = *reinterpret_cast<uint32_t*>(&h);
            } else {
                __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
                w[i] = *reinterpret_cast<uint32_t*>(&h);
            }
        }
        *reinterpret_cast<uint4*>(&o) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
#pragma unroll
        for (int e = 0; e < elem<T>::kPack; ++e) o.v[e] = elem<T>::from_f(f[e]);
    }
    return o;
}

// Unsigned 32-bit division by a run-time invariant divisor with one multiply-high and a shift
// (the round-up method of Granlund & Montgomery, "Division by invariant integers using
// multiplication", PLDI 1994): shift = ceil(log2 d), mul = floor(2^32 (2^shift - d) / d) + 1,
// n / d = (mulhi(n, mul) + n) >> shift, the sum taken in 64 bits.
struct FastDiv {
    uint32_t d = 1, mul = 0, shift = 0;
    __host__ void init(uint32_t divisor) {
        d = divisor ? divisor : 1;
        shift = 0;
        while ((1ull << shift) < d) ++shift;
        mul = static_cast<uint32_t>(((1ull << 32) * ((1ull << shift) - d)) / d + 1);
        if (d == 1) mul = 0;
    }
    __device__ __forceinline__ uint32_t div(uint32_t n) const {
        return static_cast<uint32_t>((static_cast<uint64_t>(__umulhi(n, mul)) + n) >> shift);
    }
    __device__ __forceinline__ uint32_t mod(uint32_t n) const { return n - div(n) * d; }
};

}  // namespace hc
