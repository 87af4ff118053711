// flash_attention_fwd_fused on B200.
//
// Algorithm: the reference golden's online softmax
// (ops/flash_attention_fwd_fused/golden/flash_attention_fwd_fused_golden.cpp:26-107):
// per query row keep a running max m and sum l, rescale the accumulator when m grows,
// O = acc / l; causal masking hides key k from query q when k > q (golden.cpp:61-66).
// Added output: lse = m + ln(l) per row (natural log), the standard flash-attention residual.
//
// Tensor-core path (bf16/fp16, D = D_v = 128), one persistent CTA per SM:
//   * a CTA work unit is (b*h, block of 256 query rows) = two 128-row Q tiles;
//   * warp 9 (producer) streams Q tiles and 128-key K/V tiles into shared memory with TMA
//     (128-byte swizzle, a 4-stage K/V ring, no multicast);
//   * warp 8 (one thread) issues tcgen05.mma: S_i = Q_i K^T into TMEM (M=128, N=128, K=16 x 8)
//     and O_i += P_i V with P read straight from TMEM (the "TS" form), V as an MN-major operand;
//   * warpgroups 0 and 1 each own one Q tile: thread t owns row t (TMEM lane t), reads its S row
//     with tcgen05.ld, applies the causal / sequence-tail mask, updates (m, l) in the log2
//     domain, writes P (16-bit) back over its S row with tcgen05.st, and rescales its O row in
//     TMEM only when the running max grew by more than 2^8 (lazy rescaling: exact, because O and
//     l always refer to the same m);
//   * the two Q tiles ping-pong: the tensor core runs one tile's MMAs while the other tile's
//     softmax runs on the CUDA cores;
//   * the epilogue (O / l -> 16-bit, lse) is done by the owning warpgroup from TMEM.
// TMEM: S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512) columns; P_i overlays S_i.
// Every mbarrier wait is bounded (4 s of global time): on expiry the kernel records the wait site
// in a device error word, all roles unwind, in-flight copies and MMAs are drained, TMEM is freed,
// and the host reports HC_ERR_TIMEOUT through hc_check_device_error().
//
// SIMT path: any other head dims (<= 256), fp32, or non-positive scale.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <mutex>

#include "hc_device.cuh"
#include "hc_internal.h"
#include "sm100.cuh"
#include "tmap.h"

namespace hc {
namespace fa {

using namespace sm100;

constexpr uint32_t kBM = 128;      // query rows per Q tile
constexpr uint32_t kBN = 128;      // keys per K/V tile
constexpr uint32_t kHD = 128;      // head dim (D = D_v)
constexpr uint32_t kStages = 4;    // K/V ring depth
constexpr uint32_t kThreads = 384;
constexpr uint32_t kTileBytes = kBM * kHD * 2;   // 32 KB, one 16-bit 128x128 tile
constexpr uint32_t kHalfBytes = kTileBytes / 2;  // one 64-column swizzle panel
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffKV = 2 * kTileBytes;
constexpr uint32_t kOffBar = kOffKV + kStages * kTileBytes;
constexpr uint32_t kSmemBytes = kOffBar + 256 + 1024;  // + barriers/misc + alignment slack
constexpr float kRescaleThreshold = 8.0f;              // log2 units

// Error word bits: which wait expired.
enum : uint32_t {
    kErrProducerQ = 1u << 0,
    kErrProducerKV = 1u << 1,
    kErrMmaQ = 1u << 2,
    kErrMmaKV = 1u << 3,
    kErrMmaP = 1u << 4,
    kErrSoftS = 1u << 5,
    kErrSoftO = 1u << 6,
    kErrDrain = 1u << 7,
};

__device__ uint32_t g_fa_error_word;

struct Params {
    void* o;
    float* lse;
    uint32_t S_q, S_k, BH, n_qblk, num_units;
    float scale_log2;  // softmax scale * log2(e), > 0
    uint32_t causal;
};

struct Bars {
    uint64_t q_full, q_empty;
    uint64_t kv_full[kStages], kv_empty[kStages];
    uint64_t s_full[2], p_full[2], o_full[2];
    uint64_t mma_done;
};

__device__ __forceinline__ void unit_coords(const Params& p, uint32_t u, uint32_t& bh, uint32_t& qb) {
    uint32_t r = u / p.BH;
    bh = u - r * p.BH;
    // Causal: hand out the longest query blocks first so the persistent CTAs finish together.
    qb = p.causal ? (p.n_qblk - 1 - r) : r;
}

__device__ __forceinline__ uint32_t kv_tiles_for(const Params& p, uint32_t row0) {
    uint32_t nk = (p.S_k + kBN - 1) / kBN;
    if (p.causal) {
        uint32_t lim = row0 / kBN + 1;
        if (lim < nk) nk = lim;
    }
    return nk;
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <bool kBF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    if (kBF16) {
        __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&h);
    } else {
        __half2 h = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&h);
    }
}

__device__ __forceinline__ void issue_qk(uint32_t d_tmem, uint32_t q_addr, uint32_t k_addr, uint32_t idesc) {
#pragma unroll
    for (uint32_t kk = 0; kk < kHD / 16; ++kk) {
        uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
        mma_ss(d_tmem, make_sw128_desc(q_addr + off, 16, 1024), make_sw128_desc(k_addr + off, 16, 1024), idesc, kk > 0);
    }
}

__device__ __forceinline__ void issue_pv(uint32_t o_tmem, uint32_t p_tmem, uint32_t v_addr, uint32_t idesc,
                                         bool accumulate) {
#pragma unroll
    for (uint32_t kk = 0; kk < kBN / 16; ++kk) {
        // 16 keys = 16 rows of the MN-major V panel = 2 swizzle atoms (2048 B); P: 8 columns.
        mma_ts(o_tmem, p_tmem + kk * 8, make_sw128_desc(v_addr + kk * 2048, kHalfBytes, 1024), idesc,
               (accumulate || kk > 0) ? 1u : 0u);
    }
}

template <bool kBF16>
__global__ void __launch_bounds__(kThreads, 1)
    fa_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffBar + sizeof(Bars));
    volatile uint32_t* abort_flag = tmem_slot + 1;
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        mbar_init(&bars->q_full, 1);
        mbar_init(&bars->q_empty, 1);
        for (uint32_t s = 0; s < kStages; ++s) {
            mbar_init(&bars->kv_full[s], 1);
            mbar_init(&bars->kv_empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bars->s_full[i], 1);
            mbar_init(&bars->p_full[i], 128);
            mbar_init(&bars->o_full[i], 1);
        }
        mbar_init(&bars->mma_done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 8) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    if (warp == 9 && lane == 0) {
        prefetch_tmap(&tm_q);
        prefetch_tmap(&tm_k);
        prefetch_tmap(&tm_v);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const uint32_t sQ = smem_u32(smem + kOffQ);
    const uint32_t sKV = smem_u32(smem + kOffKV);

    if (warp == 9) {
        // ===================================== producer =====================================
        if (lane == 0) {
            uint32_t stage = 0, phase = 0, q_iter = 0;
            int32_t pending[kStages];
            for (uint32_t s = 0; s < kStages; ++s) pending[s] = -1;
            int32_t q_pending = -1;
            bool ok = true;
            for (uint32_t u = blockIdx.x; u < p.num_units && ok; u += gridDim.x, ++q_iter) {
                uint32_t bh, qb;
                unit_coords(p, u, bh, qb);
                const uint32_t row0 = qb * 2 * kBM;
                const uint32_t nkv = kv_tiles_for(p, row0 + kBM);
                if (!mbar_wait_bounded(&bars->q_empty, (q_iter & 1) ^ 1, abort_flag, &g_fa_error_word, kErrProducerQ)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&bars->q_full, 2 * kTileBytes);
                for (uint32_t i = 0; i < 2; ++i)
                    for (uint32_t h = 0; h < 2; ++h)
                        tma_load_3d(smem + kOffQ + i * kTileBytes + h * kHalfBytes, &tm_q, &bars->q_full,
                                    static_cast<int32_t>(h * 64), static_cast<int32_t>(row0 + i * kBM),
                                    static_cast<int32_t>(bh));
                q_pending = static_cast<int32_t>(q_iter & 1);
                for (uint32_t j = 0; j < nkv && ok; ++j) {
                    for (uint32_t kv = 0; kv < 2; ++kv) {
                        if (!mbar_wait_bounded(&bars->kv_empty[stage], phase ^ 1, abort_flag, &g_fa_error_word,
                                               kErrProducerKV)) {
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(&bars->kv_full[stage], kTileBytes);
                        for (uint32_t h = 0; h < 2; ++h)
                            tma_load_3d(smem + kOffKV + stage * kTileBytes + h * kHalfBytes, kv ? &tm_v : &tm_k,
                                        &bars->kv_full[stage], static_cast<int32_t>(h * 64),
                                        static_cast<int32_t>(j * kBN), static_cast<int32_t>(bh));
                        pending[stage] = static_cast<int32_t>(phase);
                        if (++stage == kStages) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                }
            }
            if (!ok) {
                // Drain: every TMA copy issued must land before the CTA's shared memory is released.
                volatile uint32_t never = 0;
                for (uint32_t s = 0; s < kStages; ++s)
                    if (pending[s] >= 0)
                        mbar_wait_bounded(&bars->kv_full[s], static_cast<uint32_t>(pending[s]), &never, &g_fa_error_word,
                                          kErrDrain, 1000000000ull);
                if (q_pending >= 0)
                    mbar_wait_bounded(&bars->q_full, static_cast<uint32_t>(q_pending), &never, &g_fa_error_word,
                                      kErrDrain, 1000000000ull);
            }
        }
    } else if (warp == 8) {
        // ==================================== MMA issuer ====================================
        if (lane == 0) {
            const uint32_t idesc_qk = make_idesc_f16(kBF16, kBM, kBN, false, false);
            const uint32_t idesc_pv = make_idesc_f16(kBF16, kBM, kHD, false, true);
            const uint32_t tS[2] = {tmem_base, tmem_base + 128};
            const uint32_t tO[2] = {tmem_base + 256, tmem_base + 384};
            const uint32_t qa[2] = {sQ, sQ + kTileBytes};
            uint32_t stage = 0, phase = 0, q_iter = 0;
            uint32_t p_par[2] = {0, 0};
            bool ok = true;
            auto wait_kv = [&](uint32_t& st) -> bool {
                if (!mbar_wait_bounded(&bars->kv_full[stage], phase, abort_flag, &g_fa_error_word, kErrMmaKV))
                    return false;
                tc_fence_after();
                st = stage;
                if (++stage == kStages) {
                    stage = 0;
                    phase ^= 1;
                }
                return true;
            };
            auto wait_p = [&](int i) -> bool {
                if (!mbar_wait_bounded(&bars->p_full[i], p_par[i], abort_flag, &g_fa_error_word, kErrMmaP)) return false;
                p_par[i] ^= 1;
                tc_fence_after();
                return true;
            };
            for (uint32_t u = blockIdx.x; u < p.num_units && ok; u += gridDim.x, ++q_iter) {
                uint32_t bh, qb;
                unit_coords(p, u, bh, qb);
                const uint32_t row0 = qb * 2 * kBM;
                const uint32_t n0 = kv_tiles_for(p, row0);
                const uint32_t nkv = kv_tiles_for(p, row0 + kBM);
                if (!mbar_wait_bounded(&bars->q_full, q_iter & 1, abort_flag, &g_fa_error_word, kErrMmaQ)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                uint32_t kst, vst;
                if (!wait_kv(kst)) { ok = false; break; }
                issue_qk(tS[0], qa[0], sKV + kst * kTileBytes, idesc_qk);
                tc_commit(&bars->s_full[0]);
                issue_qk(tS[1], qa[1], sKV + kst * kTileBytes, idesc_qk);
                tc_commit(&bars->s_full[1]);
                tc_commit(&bars->kv_empty[kst]);
                if (nkv == 1) tc_commit(&bars->q_empty);
                for (uint32_t j = 1; j < nkv; ++j) {
                    if (!wait_kv(vst)) { ok = false; break; }            // V_{j-1}
                    if (j - 1 < n0) {
                        if (!wait_p(0)) { ok = false; break; }
                        issue_pv(tO[0], tS[0], sKV + vst * kTileBytes, idesc_pv, j - 1 > 0);
                    }
                    if (!wait_kv(kst)) { ok = false; break; }            // K_j
                    if (j < n0) {
                        issue_qk(tS[0], qa[0], sKV + kst * kTileBytes, idesc_qk);
                        tc_commit(&bars->s_full[0]);
                    }
                    if (!wait_p(1)) { ok = false; break; }
                    issue_pv(tO[1], tS[1], sKV + vst * kTileBytes, idesc_pv, j - 1 > 0);
                    tc_commit(&bars->kv_empty[vst]);
                    issue_qk(tS[1], qa[1], sKV + kst * kTileBytes, idesc_qk);
                    tc_commit(&bars->s_full[1]);
                    tc_commit(&bars->kv_empty[kst]);
                    if (j + 1 == nkv) tc_commit(&bars->q_empty);
                }
                if (!ok) break;
                if (!wait_kv(vst)) { ok = false; break; }                // V_{nkv-1}
                if (n0 == nkv) {
                    if (!wait_p(0)) { ok = false; break; }
                    issue_pv(tO[0], tS[0], sKV + vst * kTileBytes, idesc_pv, nkv > 1);
                }
                tc_commit(&bars->o_full[0]);
                if (!wait_p(1)) { ok = false; break; }
                issue_pv(tO[1], tS[1], sKV + vst * kTileBytes, idesc_pv, nkv > 1);
                tc_commit(&bars->o_full[1]);
                tc_commit(&bars->kv_empty[vst]);
            }
            // All issued MMAs must complete before TMEM is freed (normal and abort paths alike).
            tc_commit(&bars->mma_done);
            volatile uint32_t never = 0;
            mbar_wait_bounded(&bars->mma_done, 0, &never, &g_fa_error_word, kErrDrain, 1000000000ull);
        }
    } else if (warp < 8) {
        // ============================== softmax / epilogue ===============================
        const uint32_t wg = warp / 4;                 // Q tile owned by this warpgroup
        const uint32_t r_local = threadIdx.x - wg * 128;  // row within the tile = TMEM lane
        const uint32_t lane_field = ((warp & 3) * 32) << 16;
        const uint32_t tS = tmem_base + wg * 128 + lane_field;
        const uint32_t tO = tmem_base + 256 + wg * 128 + lane_field;
        uint32_t s_par = 0, o_par = 0;
        for (uint32_t u = blockIdx.x; u < p.num_units; u += gridDim.x) {
            uint32_t bh, qb;
            unit_coords(p, u, bh, qb);
            const uint32_t row0 = qb * 2 * kBM + wg * kBM;
            const uint32_t row = row0 + r_local;
            const uint32_t n_i = kv_tiles_for(p, row0);
            float m = -INFINITY, l = 0.f;
            bool ok = true;
            for (uint32_t j = 0; j < n_i; ++j) {
                ok = mbar_wait_bounded(&bars->s_full[wg], s_par, abort_flag, &g_fa_error_word, kErrSoftS);
                // Keep the warp converged and its decision uniform before the warp-collective
                // tcgen05 loads/stores below.
                if (!__all_sync(0xffffffffu, ok)) {
                    ok = false;
                    break;
                }
                s_par ^= 1;
                tc_fence_after();
                uint32_t sr[128];
                tmem_ld32(tS + 0, *reinterpret_cast<uint32_t(*)[32]>(sr + 0));
                tmem_ld32(tS + 32, *reinterpret_cast<uint32_t(*)[32]>(sr + 32));
                tmem_ld32(tS + 64, *reinterpret_cast<uint32_t(*)[32]>(sr + 64));
                tmem_ld32(tS + 96, *reinterpret_cast<uint32_t(*)[32]>(sr + 96));
                tmem_wait_ld();
                float* s = reinterpret_cast<float*>(sr);
                const uint32_t kbase = j * kBN;
                // Valid keys of this tile for this row: causal (k <= row) and sequence tail (k < S_k).
                int32_t lim = static_cast<int32_t>(p.S_k) - static_cast<int32_t>(kbase);
                if (p.causal) {
                    int32_t lc = static_cast<int32_t>(row) - static_cast<int32_t>(kbase) + 1;
                    if (lc < lim) lim = lc;
                }
                if (lim < static_cast<int32_t>(kBN)) {
#pragma unroll
                    for (int c = 0; c < 128; ++c) s[c] = (c < lim) ? s[c] : -INFINITY;
                }
                float mx = s[0];
#pragma unroll
                for (int c = 1; c < 128; ++c) mx = fmaxf(mx, s[c]);
                const float mx_l2 = mx * p.scale_log2;
                // Lazy rescaling: move the reference max only when it grows by more than 2^8.
                bool need = (mx_l2 > m + kRescaleThreshold);
                float alpha = 1.f;
                if (need) {
                    alpha = ex2(m - mx_l2);  // 0 on the first tile (m = -inf)
                    m = mx_l2;
                    l *= alpha;
                }
                if (j > 0 && __any_sync(0xffffffffu, need)) {
                    // O row *= alpha (PV of the previous tile has completed: it was issued
                    // before the S MMA whose completion we just waited for).
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        uint32_t orow[32];
                        tmem_ld32(tO + c * 32, orow);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 32; ++e) orow[e] = __float_as_uint(__uint_as_float(orow[e]) * alpha);
                        tmem_st32(tO + c * 32, orow);
                    }
                }
                const float neg_m = (m == -INFINITY) ? 0.f : -m;
                float lsum = 0.f;
                uint32_t pk[64];
#pragma unroll
                for (int c = 0; c < 64; ++c) {
                    float p0 = ex2(fmaf(s[2 * c], p.scale_log2, neg_m));
                    float p1 = ex2(fmaf(s[2 * c + 1], p.scale_log2, neg_m));
                    lsum += p0 + p1;
                    pk[c] = pack2<kBF16>(p0, p1);
                }
                l += lsum;
                tmem_st32(tS + 0, pk + 0);
                tmem_st32(tS + 32, pk + 32);
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(&bars->p_full[wg]);
            }
            if (!ok) break;
            // ---- epilogue ----
            ok = mbar_wait_bounded(&bars->o_full[wg], o_par, abort_flag, &g_fa_error_word, kErrSoftO);
            if (!__all_sync(0xffffffffu, ok)) break;
            o_par ^= 1;
            tc_fence_after();
            const float inv_l = 1.0f / l;
            const bool in_range = row < p.S_q;
            uint8_t* orow_g = static_cast<uint8_t*>(p.o) + (static_cast<size_t>(bh) * p.S_q + row) * kHD * 2;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint32_t orow[32];
                tmem_ld32(tO + c * 32, orow);
                tmem_wait_ld();
                uint32_t packed[16];
#pragma unroll
                for (int e = 0; e < 16; ++e)
                    packed[e] = pack2<kBF16>(__uint_as_float(orow[2 * e]) * inv_l, __uint_as_float(orow[2 * e + 1]) * inv_l);
                if (in_range) {
                    uint4* dst = reinterpret_cast<uint4*>(orow_g + c * 64);
#pragma unroll
                    for (int v = 0; v < 4; ++v)
                        dst[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
                }
            }
            if (in_range && p.lse) p.lse[static_cast<size_t>(bh) * p.S_q + row] = (m + __log2f(l)) * 0.6931471805599453f;
            tc_fence_before();
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 8) {
        __syncwarp();
        tmem_dealloc(tmem_base, 512);
    }
}

// ======================================================================================
// SIMT path: one warp per query row; lanes score 32 keys at a time, then accumulate
// D_v / 32 output columns each.  fp32 math, any D, D_v <= 256.
// ======================================================================================
template <typename T>
__global__ void __launch_bounds__(256) fa_fwd_simt_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                          const T* __restrict__ v, T* __restrict__ o,
                                                          float* __restrict__ lse, uint32_t BH, uint32_t S_q,
                                                          uint32_t S_k, uint32_t D, uint32_t Dv, float scale,
                                                          uint32_t causal) {
    constexpr int kMaxD = 256;
    __shared__ float qs[8][kMaxD];
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const uint64_t total_rows = static_cast<uint64_t>(BH) * S_q;
    for (uint64_t gr = static_cast<uint64_t>(blockIdx.x) * 8 + warp; gr < total_rows;
         gr += static_cast<uint64_t>(gridDim.x) * 8) {
        const uint64_t bh = gr / S_q;
        const uint32_t qi = static_cast<uint32_t>(gr % S_q);
        const T* qrow = q + gr * D;
        for (uint32_t d = lane; d < D; d += 32) qs[warp][d] = elem<T>::to_f(qrow[d]);
        __syncwarp();
        float m = -INFINITY, l = 0.f;
        float acc[kMaxD / 32];
#pragma unroll
        for (int i = 0; i < kMaxD / 32; ++i) acc[i] = 0.f;
        const uint32_t kend = causal ? min(S_k, qi + 1) : S_k;
        for (uint32_t k0 = 0; k0 < kend; k0 += 32) {
            const uint32_t kj = k0 + lane;
            float sc = -INFINITY;
            if (kj < kend) {
                const T* krow = k + (bh * S_k + kj) * D;
                float dot = 0.f;
                for (uint32_t d = 0; d < D; ++d) dot = fmaf(qs[warp][d], elem<T>::to_f(krow[d]), dot);
                sc = dot * scale;
            }
            float cmax = sc;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, off));
            const float m_new = fmaxf(m, cmax);
            const float alpha = (m == -INFINITY) ? 0.f : expf(m - m_new);
            const float pj = (kj < kend) ? expf(sc - m_new) : 0.f;
            float psum = warp_sum(pj);
            l = l * alpha + psum;
#pragma unroll
            for (int i = 0; i < kMaxD / 32; ++i) acc[i] *= alpha;
            const uint32_t cnt = min(32u, kend - k0);
            for (uint32_t jj = 0; jj < cnt; ++jj) {
                const float pv = __shfl_sync(0xffffffffu, pj, jj);
                const T* vrow = v + (bh * S_k + k0 + jj) * Dv;
#pragma unroll
                for (int i = 0; i < kMaxD / 32; ++i) {
                    uint32_t d = lane + 32 * i;
                    if (d < Dv) acc[i] = fmaf(pv, elem<T>::to_f(vrow[d]), acc[i]);
                }
            }
            m = m_new;
        }
        T* orow = o + gr * Dv;
#pragma unroll
        for (int i = 0; i < kMaxD / 32; ++i) {
            uint32_t d = lane + 32 * i;
            if (d < Dv) orow[d] = elem<T>::from_f(acc[i] / l);
        }
        if (lse && lane == 0) lse[gr] = m + logf(l);
        __syncwarp();
    }
}

// Self-test of the bounded-wait machinery: one CTA waits on an mbarrier that nothing arrives on.
// The wait must give up after `budget_ns`, record the site in the error word and let the kernel
// exit normally (no trap, no hang).
__global__ void bounded_wait_selftest_kernel(uint64_t budget_ns) {
    __shared__ uint64_t bar;
    __shared__ volatile uint32_t abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0)
        mbar_wait_bounded(&bar, 0, &abort_flag, &g_fa_error_word, kErrDrain << 1, budget_ns);
    __syncthreads();
}

uint32_t read_error_word(const char** name) {
    *name = "flash_attention_fwd_fused";
    uint32_t word = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&word, g_fa_error_word, sizeof(word)) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (word) cudaMemcpyToSymbol(g_fa_error_word, &zero, sizeof(zero));
    return word;
}

thread_local int t_last_path = 0;

template <bool kBF16>
int launch_tc(const void* q, const void* k, const void* v, void* o, float* lse,
              const flash_attention_fwd_fused_tiling_data* t, cudaStream_t stream) {
    static std::once_flag reg_once;
    std::call_once(reg_once, [] { register_error_word(read_error_word); });
    const uint64_t BH = static_cast<uint64_t>(t->B) * t->H;
    CUtensorMap tmq, tmk, tmv;
    const CUtensorMapDataType dt = kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const uint32_t box[3] = {64, 128, 1};
    {
        uint64_t dims[3] = {kHD, t->S_q, BH};
        uint64_t strides[2] = {kHD * 2, static_cast<uint64_t>(t->S_q) * kHD * 2};
        int rc = encode_tmap(&tmq, dt, 3, q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    {
        uint64_t dims[3] = {kHD, t->S_k, BH};
        uint64_t strides[2] = {kHD * 2, static_cast<uint64_t>(t->S_k) * kHD * 2};
        int rc = encode_tmap(&tmk, dt, 3, k, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
        rc = encode_tmap(&tmv, dt, 3, v, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    Params prm;
    prm.o = o;
    prm.lse = lse;
    prm.S_q = t->S_q;
    prm.S_k = t->S_k;
    prm.BH = static_cast<uint32_t>(BH);
    prm.n_qblk = (t->S_q + 2 * kBM - 1) / (2 * kBM);
    uint64_t units = BH * prm.n_qblk;
    if (units > 0xffffffffull) return fail(HC_ERR_UNSUPPORTED, "flash_attention: too many work units");
    prm.num_units = static_cast<uint32_t>(units);
    prm.scale_log2 = t->scale * 1.4426950408889634f;
    prm.causal = t->maskType;
    static bool attr_set[2] = {false, false};
    if (!attr_set[kBF16]) {
        cudaError_t e = cudaFuncSetAttribute(fa_fwd_tc_kernel<kBF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kSmemBytes));
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(fa_fwd_tc_kernel)");
        attr_set[kBF16] = true;
    }
    uint32_t grid = static_cast<uint32_t>(sm_count());
    if (grid > prm.num_units) grid = prm.num_units;
    fa_fwd_tc_kernel<kBF16><<<grid, kThreads, kSmemBytes, stream>>>(tmq, tmk, tmv, prm);
    t_last_path = 1;
    return check_launch("fa_fwd_tc_kernel");
}

template <typename T>
int launch_simt(const void* q, const void* k, const void* v, void* o, float* lse,
                const flash_attention_fwd_fused_tiling_data* t, cudaStream_t stream) {
    const uint64_t rows = static_cast<uint64_t>(t->B) * t->H * t->S_q;
    uint64_t blocks = (rows + 7) / 8;
    uint64_t cap = static_cast<uint64_t>(sm_count()) * 8;
    if (blocks > cap) blocks = cap;
    fa_fwd_simt_kernel<T><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
        static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(v), static_cast<T*>(o), lse,
        t->B * t->H, t->S_q, t->S_k, t->D, t->D_v, t->scale, t->maskType);
    t_last_path = 2;
    return check_launch("fa_fwd_simt_kernel");
}

}  // namespace fa
}  // namespace hc

using namespace hc;

extern "C" int hc_flash_attention_fwd_fused_launch(const void* q, const void* k, const void* v, void* o, float* lse,
                                                   const flash_attention_fwd_fused_tiling_data* t, int dtype,
                                                   void* stream) {
    if (!t) return fail(HC_ERR_INVALID, "flash_attention: null tiling");
    if (t->B == 0 || t->H == 0 || t->S_q == 0) return ok();
    if (!q || !k || !v || !o) return fail(HC_ERR_INVALID, "flash_attention: null pointer");
    if (t->S_k == 0) return fail(HC_ERR_INVALID, "flash_attention: S_k must be >= 1");
    if (t->D == 0 || t->D_v == 0 || t->D > 256 || t->D_v > 256)
        return fail(HC_ERR_UNSUPPORTED, "flash_attention: D=%u D_v=%u (1..256 supported)", t->D, t->D_v);
    if (t->maskType > 1) return fail(HC_ERR_INVALID, "flash_attention: maskType %u (0 none, 1 causal)", t->maskType);
    if (!std::isfinite(t->scale)) return fail(HC_ERR_INVALID, "flash_attention: scale must be finite");
    if (fault_hit("launch")) return fail(HC_ERR_INJECTED, "flash_attention: injected launch failure");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool tc_shape = t->D == fa::kHD && t->D_v == fa::kHD && t->scale > 0.f &&
                          aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o);
    if (dtype == HC_DTYPE_BF16) {
        if (tc_shape) return fa::launch_tc<true>(q, k, v, o, lse, t, s);
        return fa::launch_simt<bf16_t>(q, k, v, o, lse, t, s);
    }
    if (dtype == HC_DTYPE_F16) {
        if (tc_shape) return fa::launch_tc<false>(q, k, v, o, lse, t, s);
        return fa::launch_simt<f16_t>(q, k, v, o, lse, t, s);
    }
    if (dtype == HC_DTYPE_F32) return fa::launch_simt<float>(q, k, v, o, lse, t, s);
    return fail(HC_ERR_UNSUPPORTED, "flash_attention: dtype %d not supported (BF16, F16, F32)", dtype);
}

extern "C" int hc_flash_attention_last_path(void) { return fa::t_last_path; }

extern "C" int hc_selftest_bounded_wait(uint32_t budget_us) {
    static std::once_flag reg_once;
    std::call_once(reg_once, [] { register_error_word(fa::read_error_word); });
    if (budget_us == 0 || budget_us > 1000000) return fail(HC_ERR_INVALID, "budget_us must be in 1..1000000");
    fa::bounded_wait_selftest_kernel<<<1, 32>>>(static_cast<uint64_t>(budget_us) * 1000ull);
    int rc = check_launch("bounded_wait_selftest_kernel");
    if (rc) return rc;
    HC_CHECK_CUDA(cudaDeviceSynchronize());
    return hc_check_device_error();
}
