// CPU restatement of the reference harness's goldens -- TEST INFRASTRUCTURE ONLY (see oracle.h).
//
// Every function restates one golden of z-zijie/ascend-npu-harness step for step, including its
// accumulation precision (fp64 where the golden uses double) and operation order, so that on the
// same inputs the results are bit-identical to the golden compiled from the reference sources.
// Built with -ffp-contract=off so no multiply-add is fused (the goldens are compiled for a
// baseline x86-64 target, which has no FMA).
#include "oracle.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <random>
#include <thread>
#include <vector>

extern "C" {

// ------------------------------------------------------------------------------------------
// generators
// ------------------------------------------------------------------------------------------
// include/harness/test_utils.hpp:39-46
void oracle_uniform_f32(float* out, size_t n, uint64_t seed, float lo, float hi) {
    std::mt19937_64 gen(seed);
    std::uniform_real_distribution<float> dist(lo, hi);
    for (size_t i = 0; i < n; ++i) out[i] = dist(gen);
}

void oracle_normal_f32(float* out, size_t n, uint64_t seed, float mean, float stddev) {
    std::mt19937_64 gen(seed);
    const double two_pi = 6.283185307179586476925286766559;
    size_t i = 0;
    while (i < n) {
        // u1 in (0, 1], u2 in [0, 1) from the top 53 bits of each draw.
        double u1 = 1.0 - static_cast<double>(gen() >> 11) * 0x1.0p-53;
        double u2 = static_cast<double>(gen() >> 11) * 0x1.0p-53;
        double r = std::sqrt(-2.0 * std::log(u1));
        out[i++] = static_cast<float>(mean + stddev * r * std::cos(two_pi * u2));
        if (i < n) out[i++] = static_cast<float>(mean + stddev * r * std::sin(two_pi * u2));
    }
}

// include/harness/test_utils.hpp:59-72 (float arithmetic, std::pow/cos/sin on floats)
void oracle_rope_cos_sin(size_t seq_len, size_t half, float* cos_out, float* sin_out, float base) {
    for (size_t s = 0; s < seq_len; ++s) {
        for (size_t d = 0; d < half; ++d) {
            float expo = 2.0f * static_cast<float>(d) / static_cast<float>(half * 2);
            float theta = static_cast<float>(s) / std::pow(base, expo);
            cos_out[s * half + d] = std::cos(theta);
            sin_out[s * half + d] = std::sin(theta);
        }
    }
}

// ------------------------------------------------------------------------------------------
// 16-bit codecs: correctly rounded (round-half-to-even) narrowing, exact widening.
// ------------------------------------------------------------------------------------------
static inline uint32_t f2u(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return u;
}
static inline float u2f(uint32_t u) {
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

void oracle_f32_to_bf16(const float* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        uint32_t u = f2u(in[i]);
        if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) {
            out[i] = static_cast<uint16_t>((u >> 16) | 0x0040u);  // quiet NaN
            continue;
        }
        uint32_t lsb = (u >> 16) & 1u;
        out[i] = static_cast<uint16_t>((u + 0x7fffu + lsb) >> 16);
    }
}

void oracle_bf16_to_f32(const uint16_t* in, float* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = u2f(static_cast<uint32_t>(in[i]) << 16);
}

void oracle_f32_to_f16(const float* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        uint32_t u = f2u(in[i]);
        uint16_t sign = static_cast<uint16_t>((u >> 16) & 0x8000u);
        uint32_t a = u & 0x7fffffffu;
        if (a >= 0x7f800000u) {  // inf / nan
            out[i] = static_cast<uint16_t>(sign | 0x7c00u | (a > 0x7f800000u ? 0x0200u : 0u));
            continue;
        }
        // 65520 and above round to infinity.
        if (a >= 0x477ff000u) {
            out[i] = static_cast<uint16_t>(sign | 0x7c00u);
            continue;
        }
        int32_t e = static_cast<int32_t>(a >> 23) - 127;
        if (e >= -14) {  // normal half
            uint32_t mant = a & 0x7fffffu;
            uint32_t h = (static_cast<uint32_t>(e + 15) << 10) | (mant >> 13);
            uint32_t rem = mant & 0x1fffu;
            if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1;  // carries into exponent correctly
            out[i] = static_cast<uint16_t>(sign | h);
        } else {  // subnormal half (or zero): value = m * 2^-24
            if (e < -25) {
                out[i] = sign;
                continue;
            }
            uint32_t mant = (a & 0x7fffffu) | 0x800000u;  // 24-bit significand, value = mant * 2^(e-23)
            int shift = -e - 1;                             // mant * 2^(e-23) / 2^-24 = mant >> (-(e+1))
            uint32_t h = mant >> shift;
            uint32_t rem = mant & ((1u << shift) - 1u);
            uint32_t halfway = 1u << (shift - 1);
            if (rem > halfway || (rem == halfway && (h & 1u))) h += 1;
            out[i] = static_cast<uint16_t>(sign | h);
        }
    }
}

void oracle_f16_to_f32(const uint16_t* in, float* out, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        uint32_t h = in[i];
        uint32_t sign = (h & 0x8000u) << 16;
        uint32_t e = (h >> 10) & 0x1fu;
        uint32_t m = h & 0x3ffu;
        float v;
        if (e == 0) {
            v = std::ldexp(static_cast<float>(m), -24);
            out[i] = u2f(f2u(v) | sign);
            continue;
        }
        if (e == 31) {
            out[i] = u2f(sign | 0x7f800000u | (m << 13));
            continue;
        }
        out[i] = u2f(sign | ((e - 15 + 127) << 23) | (m << 13));
    }
}

// ------------------------------------------------------------------------------------------
// elementwise family
// ------------------------------------------------------------------------------------------
void oracle_elementwise_add(const float* x, const float* y, float* z, size_t n) {
    for (size_t i = 0; i < n; ++i) z[i] = x[i] + y[i];
}

void oracle_axpy_scalar_affine(const float* x, float* y, size_t n, float alpha, float beta) {
    for (size_t i = 0; i < n; ++i) y[i] = alpha * x[i] + beta;
}

void oracle_broadcast_binary(const float* x, const float* y, const float* bias, float* z, int64_t B, int64_t C,
                             int64_t H, int64_t W, int64_t y_batch) {
    const int64_t plane = H * W;
    for (int64_t b = 0; b < B; ++b) {
        const float* yb = y + (y_batch == 1 ? 0 : b) * C;
        for (int64_t c = 0; c < C; ++c) {
            const float s = yb[c], t = bias[c];
            const int64_t base = (b * C + c) * plane;
            for (int64_t i = 0; i < plane; ++i) z[base + i] = x[base + i] * s + t;
        }
    }
}

void oracle_activation_gelu_silu(const float* x, float* y, size_t n, int act) {
    const float k0 = 0.7978845608f, k1 = 0.044715f;
    for (size_t i = 0; i < n; ++i) {
        const float v = x[i];
        if (act == 0) {
            float cube = v * v * v;
            float t = std::tanh(k0 * (v + k1 * cube));
            y[i] = 0.5f * v * (1.0f + t);
        } else if (v >= 0.0f) {
            y[i] = v / (1.0f + std::exp(-v));
        } else {
            float e = std::exp(v);
            y[i] = v * e / (1.0f + e);
        }
    }
}

void oracle_reduce_sum_lastdim(const float* x, float* out, int64_t batches, int64_t M, int64_t K) {
    for (int64_t r = 0; r < batches * M; ++r) {
        const float* row = x + r * K;
        float s = 0.0f, c = 0.0f;  // Kahan sum and compensation
        for (int64_t k = 0; k < K; ++k) {
            float yk = row[k] - c;
            float t = s + yk;
            c = (t - s) - yk;
            s = t;
        }
        out[r] = s;
    }
}

void oracle_transpose(const void* in, void* out, int mode, int64_t d0, int64_t d1, int64_t d2, int64_t d3,
                      int elem_bytes) {
    // Reduce every mode to `batch` row-major R x C matrices transposed to C x R.
    int64_t batch = 1, R = d0, C = d1;
    if (mode == 1) {        // NCHW -> NHWC : per n, [C][H*W] -> [H*W][C]
        batch = d0; R = d1; C = d2 * d3;
    } else if (mode == 2) { // NHWC -> NCHW : per n, [H*W][C] -> [C][H*W]
        batch = d0; R = d2 * d3; C = d1;
    }
    const uint8_t* src = static_cast<const uint8_t*>(in);
    uint8_t* dst = static_cast<uint8_t*>(out);
    const size_t es = static_cast<size_t>(elem_bytes);
    for (int64_t b = 0; b < batch; ++b)
        for (int64_t r = 0; r < R; ++r)
            for (int64_t c = 0; c < C; ++c)
                std::memcpy(dst + ((b * C + c) * R + r) * es, src + ((b * R + r) * C + c) * es, es);
}

// ------------------------------------------------------------------------------------------
// row normalisations
// ------------------------------------------------------------------------------------------
void oracle_layer_norm(const float* x, const float* gamma, const float* beta, float* y, int64_t rows,
                       int64_t last_dim, float eps) {
    for (int64_t r = 0; r < rows; ++r) {
        const float* xr = x + r * last_dim;
        float* yr = y + r * last_dim;
        double acc = 0.0;
        for (int64_t d = 0; d < last_dim; ++d) acc += static_cast<double>(xr[d]);
        const float mean = static_cast<float>(acc / static_cast<double>(last_dim));
        double sq = 0.0;
        for (int64_t d = 0; d < last_dim; ++d) {
            float dev = xr[d] - mean;
            sq += static_cast<double>(dev * dev);
        }
        const float var = static_cast<float>(sq / static_cast<double>(last_dim));
        const float inv_std = 1.0f / std::sqrt(var + eps);
        for (int64_t d = 0; d < last_dim; ++d) {
            float nrm = (xr[d] - mean) * inv_std;
            yr[d] = nrm * gamma[d] + beta[d];
        }
    }
}

void oracle_rms_norm_rope(const float* x, const float* weight, const float* cos_t, const float* sin_t, float* out,
                          int64_t rows, int64_t H, int64_t rot, float eps, int64_t heads, int64_t S, int style) {
    const int64_t half = rot / 2;
    std::vector<float> yv(static_cast<size_t>(H));
    for (int64_t r = 0; r < rows; ++r) {
        const float* xr = x + r * H;
        float* orow = out + r * H;
        double ss = 0.0;
        for (int64_t d = 0; d < H; ++d) {
            double v = static_cast<double>(xr[d]);
            ss += v * v;
        }
        const float rms = static_cast<float>(std::sqrt(ss / static_cast<double>(H) + static_cast<double>(eps)));
        for (int64_t d = 0; d < H; ++d) yv[d] = (xr[d] / rms) * weight[d];
        const int64_t s_pos = (r / heads) % S;
        const float* cs = cos_t + s_pos * half;
        const float* sn = sin_t + s_pos * half;
        for (int64_t d = 0; d < H; ++d) orow[d] = yv[d];
        for (int64_t i = 0; i < half; ++i) {
            const int64_t a = (style == 0) ? 2 * i : i;
            const int64_t b = (style == 0) ? 2 * i + 1 : i + half;
            const float c = cs[i], z = sn[i];
            orow[a] = yv[a] * c - yv[b] * z;
            orow[b] = yv[a] * z + yv[b] * c;
        }
    }
}

// ------------------------------------------------------------------------------------------
// matmul_bias
// ------------------------------------------------------------------------------------------
void oracle_matmul_bias(const float* A, const float* B, const float* bias, float* C, int64_t M, int64_t K,
                        int64_t N) {
    for (int64_t m = 0; m < M; ++m) {
        const float* a = A + m * K;
        for (int64_t n = 0; n < N; ++n) {
            double acc = 0.0;
            for (int64_t k = 0; k < K; ++k) acc += static_cast<double>(a[k]) * static_cast<double>(B[k * N + n]);
            float v = static_cast<float>(acc);
            if (bias) v += bias[n];
            C[m * N + n] = v;
        }
    }
}

// ------------------------------------------------------------------------------------------
// flash attention forward: online softmax over 128-key tiles in fp64 (golden.cpp:26-107)
// ------------------------------------------------------------------------------------------
static void fa_heads(const float* Q, const float* K, const float* V, float* O, float* lse, int64_t h_begin,
                     int64_t h_end, int64_t S_q, int64_t S_k, int64_t D, int64_t Dv, float scale, int mask) {
    const int64_t kTile = 128;
    const double kNegBig = -1e30;  // the golden's "effectively -inf"
    std::vector<double> acc(static_cast<size_t>(Dv));
    std::vector<double> sc(static_cast<size_t>(kTile));
    for (int64_t bh = h_begin; bh < h_end; ++bh) {
        const float* Qh = Q + bh * S_q * D;
        const float* Kh = K + bh * S_k * D;
        const float* Vh = V + bh * S_k * Dv;
        for (int64_t qi = 0; qi < S_q; ++qi) {
            const float* q = Qh + qi * D;
            double m = kNegBig, l = 0.0;
            std::fill(acc.begin(), acc.end(), 0.0);
            for (int64_t k0 = 0; k0 < S_k; k0 += kTile) {
                const int64_t nk = std::min(kTile, S_k - k0);
                double m_new = m;
                for (int64_t j = 0; j < nk; ++j) {
                    const float* kr = Kh + (k0 + j) * D;
                    double dot = 0.0;
                    for (int64_t d = 0; d < D; ++d) dot += static_cast<double>(q[d]) * static_cast<double>(kr[d]);
                    double s = dot * static_cast<double>(scale);
                    if (mask == 1 && k0 + j > qi) s = kNegBig;
                    sc[j] = s;
                    if (s > m_new) m_new = s;
                }
                double l_new = l * std::exp(m - m_new);
                for (int64_t j = 0; j < nk; ++j) l_new += std::exp(sc[j] - m_new);
                const double rescale = std::exp(m - m_new);
                for (int64_t dv = 0; dv < Dv; ++dv) {
                    double a = acc[dv] * rescale;
                    for (int64_t j = 0; j < nk; ++j) a += std::exp(sc[j] - m_new) * static_cast<double>(Vh[(k0 + j) * Dv + dv]);
                    acc[dv] = a;
                }
                m = m_new;
                l = l_new;
            }
            float* o = O + (bh * S_q + qi) * Dv;
            for (int64_t dv = 0; dv < Dv; ++dv) o[dv] = static_cast<float>(acc[dv] / l);
            if (lse) lse[bh * S_q + qi] = static_cast<float>(m + std::log(l));
        }
    }
}

// ------------------------------------------------------------------------------------------
// flash attention backward (no reference golden exists: the harness has no backward).  The
// exact gradients of O = softmax(Q K^T * scale [+ causal mask]) V in fp64 for given dO:
//   P = softmax(S) row-wise, dV = P^T dO, dP = dO V^T, Delta = rowsum(P * dP) (= rowsum(dO * O)),
//   dS = P * (dP - Delta), dQ = scale * dS K, dK = scale * dS^T Q.
// ------------------------------------------------------------------------------------------
void oracle_flash_attention_bwd(const float* Q, const float* K, const float* V, const float* dO, float* dQ, float* dK,
                                float* dV, int64_t B, int64_t H, int64_t S_q, int64_t S_k, int64_t D, int64_t D_v,
                                float scale, int mask) {
    std::vector<double> p(static_cast<size_t>(S_k)), dp(static_cast<size_t>(S_k));
    std::vector<double> gk(static_cast<size_t>(S_k * D)), gv(static_cast<size_t>(S_k * D_v));
    for (int64_t bh = 0; bh < B * H; ++bh) {
        const float* Qh = Q + bh * S_q * D;
        const float* Kh = K + bh * S_k * D;
        const float* Vh = V + bh * S_k * D_v;
        const float* dOh = dO + bh * S_q * D_v;
        std::fill(gk.begin(), gk.end(), 0.0);
        std::fill(gv.begin(), gv.end(), 0.0);
        for (int64_t r = 0; r < S_q; ++r) {
            const int64_t nk = (mask == 1) ? std::min(S_k, r + 1) : S_k;
            double mx = -1e300;
            for (int64_t k = 0; k < nk; ++k) {
                double dot = 0.0;
                for (int64_t d = 0; d < D; ++d) dot += static_cast<double>(Qh[r * D + d]) * Kh[k * D + d];
                p[k] = dot * scale;
                mx = std::max(mx, p[k]);
            }
            double l = 0.0;
            for (int64_t k = 0; k < nk; ++k) {
                p[k] = std::exp(p[k] - mx);
                l += p[k];
            }
            double delta = 0.0;
            for (int64_t k = 0; k < nk; ++k) {
                p[k] /= l;
                double dot = 0.0;
                for (int64_t d = 0; d < D_v; ++d) dot += static_cast<double>(dOh[r * D_v + d]) * Vh[k * D_v + d];
                dp[k] = dot;
                delta += p[k] * dot;
            }
            for (int64_t d = 0; d < D; ++d) {
                double g = 0.0;
                for (int64_t k = 0; k < nk; ++k) g += p[k] * (dp[k] - delta) * Kh[k * D + d];
                dQ[(bh * S_q + r) * D + d] = static_cast<float>(g * scale);
            }
            for (int64_t k = 0; k < nk; ++k) {
                const double ds = p[k] * (dp[k] - delta) * scale;
                for (int64_t d = 0; d < D; ++d) gk[k * D + d] += ds * Qh[r * D + d];
                for (int64_t d = 0; d < D_v; ++d) gv[k * D_v + d] += p[k] * dOh[r * D_v + d];
            }
        }
        for (int64_t i = 0; i < S_k * D; ++i) dK[bh * S_k * D + i] = static_cast<float>(gk[i]);
        for (int64_t i = 0; i < S_k * D_v; ++i) dV[bh * S_k * D_v + i] = static_cast<float>(gv[i]);
    }
}

void oracle_flash_attention_fwd(const float* Q, const float* K, const float* V, float* O, float* lse, int64_t B,
                                int64_t H, int64_t S_q, int64_t S_k, int64_t D, int64_t D_v, float scale, int mask) {
    fa_heads(Q, K, V, O, lse, 0, B * H, S_q, S_k, D, D_v, scale, mask);
}

void oracle_flash_attention_fwd_mt(const float* Q, const float* K, const float* V, float* O, float* lse, int64_t B,
                                   int64_t H, int64_t S_q, int64_t S_k, int64_t D, int64_t D_v, float scale, int mask,
                                   int threads) {
    const int64_t BH = B * H;
    if (threads < 1) threads = 1;
    if (threads > BH) threads = static_cast<int>(BH);
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; ++t) {
        int64_t h0 = BH * t / threads, h1 = BH * (t + 1) / threads;
        pool.emplace_back(fa_heads, Q, K, V, O, lse, h0, h1, S_q, S_k, D, D_v, scale, mask);
    }
    for (auto& th : pool) th.join();
}

}  // extern "C"
