// The FMA-pipe exponential shared by the attention kernels (forward softmax, backward P).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace hc {

// 2^x for a pair, on the FMA pipe (offloads the MUFU unit, which would otherwise do as much work
// per tile as the tensor core).  Range reduction x = n + f with n = rint(x) obtained by adding
// 1.5*2^23 (the rounded integer lands in the low mantissa bits), f in [-1/2, 1/2]; 2^f by a cubic
// whose coefficients are the minimax-relative-error fit on [-1/2, 1/2] from the Remez exchange
// algorithm (max relative error 7.5e-5, below bf16's 2^-9; derivation: tests/exp2_poly_fit.py);
// 2^n applied by adding n to the exponent field.  Inputs are clamped to >= -120 so the exponent
// never underflows; callers only use it where x <= 8.5.
constexpr float kExp2C0 = 0.99992805719375610f;
constexpr float kExp2C1 = 0.69326096773147583f;
constexpr float kExp2C2 = 0.24261112511157990f;
constexpr float kExp2C3 = 0.05517166852951050f;

// bits(p) + bits(t) * 2^23 as one integer multiply-add (FMA pipe, not the ALU).
__device__ __forceinline__ float add_exponent(float p, float t) {
    uint32_t r;
    asm("mad.lo.u32 %0, %1, 8388608, %2;" : "=r"(r) : "r"(__float_as_uint(t)), "r"(__float_as_uint(p)));
    return __uint_as_float(r);
}

__device__ __forceinline__ float2 exp2_poly2(float2 x) {
    const float2 kMagic2 = make_float2(12582912.0f, 12582912.0f);  // 1.5 * 2^23
    const float2 kNegMagic2 = make_float2(-12582912.0f, -12582912.0f);
    const float2 kMinus1 = make_float2(-1.f, -1.f);
    x.x = fmaxf(x.x, -120.f);
    x.y = fmaxf(x.y, -120.f);
    const float2 t = __fadd2_rn(x, kMagic2);                    // rint(x) in the low mantissa bits
    const float2 f = __ffma2_rn(__fadd2_rn(t, kNegMagic2), kMinus1, x);  // x - rint(x)
    float2 p = __ffma2_rn(make_float2(kExp2C3, kExp2C3), f, make_float2(kExp2C2, kExp2C2));
    p = __ffma2_rn(p, f, make_float2(kExp2C1, kExp2C1));
    p = __ffma2_rn(p, f, make_float2(kExp2C0, kExp2C0));
    return make_float2(add_exponent(p.x, t.x), add_exponent(p.y, t.y));
}

}  // namespace hc
