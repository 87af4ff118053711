// Input generation for the C++ parity tests: the oracle's restatement of the harness generator
// (mt19937_64 + uniform_real_distribution<float>, include/harness/test_utils.hpp:39-46), its
// Box-Muller normal generator and its round-to-nearest-even 16-bit codecs.  Test infrastructure.
#pragma once

#include <cstdint>
#include <vector>

#include "oracle.h"

namespace hc_test {

constexpr uint64_t kSeed = 20260522;  // include/harness/test_utils.hpp:20

inline std::vector<float> uniform(size_t n, uint64_t seed, float lo = -1.0f, float hi = 1.0f) {
    std::vector<float> v(n);
    if (n) oracle_uniform_f32(v.data(), n, seed, lo, hi);
    return v;
}

inline std::vector<float> normal(size_t n, uint64_t seed) {
    std::vector<float> v(n);
    if (n) oracle_normal_f32(v.data(), n, seed, 0.0f, 1.0f);
    return v;
}

inline std::vector<uint16_t> to_bf16(const std::vector<float>& x) {
    std::vector<uint16_t> b(x.size());
    if (!x.empty()) oracle_f32_to_bf16(x.data(), b.data(), x.size());
    return b;
}

inline std::vector<float> from_bf16(const std::vector<uint16_t>& b) {
    std::vector<float> x(b.size());
    if (!b.empty()) oracle_bf16_to_f32(b.data(), x.data(), b.size());
    return x;
}

// The value a bf16 buffer holds after round-to-nearest-even quantisation of x.
inline std::vector<float> quantize_bf16(const std::vector<float>& x) { return from_bf16(to_bf16(x)); }

inline size_t prod(std::initializer_list<int64_t> dims) {
    size_t n = 1;
    for (int64_t d : dims) n *= static_cast<size_t>(d);
    return n;
}

}  // namespace hc_test
