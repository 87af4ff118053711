// Device-side helpers shared by the bandwidth-bound operator kernels: element conversions,
// 16-byte packs, streaming loads/stores and warp reductions.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

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

}  // namespace hc
