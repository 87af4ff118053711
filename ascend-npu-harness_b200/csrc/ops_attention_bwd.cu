// flash_attention backward on B200: dQ, dK, dV of O = softmax(Q K^T * scale [+ causal mask]) V
// from Q, K, V, O, dO and the forward's lse (natural log).  The harness has no backward (its
// ladder is forward only); the math is the standard one:
//   P = exp(S * scale - lse), dV = P^T dO, dP = dO V^T, Delta = rowsum(dO * O),
//   dS = P * (dP - Delta), dQ = scale * dS K, dK = scale * dS^T Q.
//
// Tensor-core path (bf16/fp16, D = D_v = 128, 16-byte aligned buffers), two kernels that reuse the
// forward's operand forms (SS Q K^T-style products with both operands K-major, TS products with
// the 16-bit operand read from TMEM and an MN-major shared-memory operand):
//   * fa_bwd_dq_kernel: a CTA per 128-row query block (rows on TMEM lanes).  It first computes
//     Delta for its rows (dO from shared memory, O from global), then for every visible 128-key
//     block j: S = Q K_j^T and dP = dO V_j^T into TMEM, dS (16-bit) over S, dQ += dS K_j.
//     It writes dQ and Delta (the [B, H, S_q] fp32 buffer the caller provides).
//   * fa_bwd_dkdv_kernel: a CTA per 128-key block (keys on TMEM lanes), launched after the dQ
//     kernel: for every query block i that sees the keys: S^T = K Q_i^T and dP^T = V dO_i^T,
//     P^T and dS^T (16-bit) over them, dV += P^T dO_i and dK += dS^T Q_i, accumulated in TMEM
//     (S^T, dP^T, dV, dK = 512 columns) and written once at the end.
// Roles per CTA: warps 0-3 the elementwise work (one TMEM lane = one row or key per thread),
// warp 4 issues tcgen05.mma, warp 5 issues TMA (no multicast).  Work units are handed out as
// complementary block pairs (b, n-1-b) of one head so that every CTA gets the same causal work.
// Every mbarrier wait is bounded as in the forward kernel.
//
// SIMT path: fp32, or any other head dims (<= 256): a warp per query row for dQ/Delta and a
// warp per key row for dK/dV, fp32 math.
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
namespace fab {

using namespace sm100;

constexpr uint32_t kBlk = 128;                  // rows (queries or keys) per block
constexpr uint32_t kPanelBytes = 128 * 64 * 2;  // one 64-column swizzle panel of a 128-row tile: 16 KB
constexpr uint32_t kTileBytes = 2 * kPanelBytes;  // a 128 x 128 16-bit tile: 32 KB
constexpr uint32_t kThreads = 192;
constexpr uint32_t kStages = 4;                 // streamed-tile ring
constexpr uint32_t kOffFixed = 0;               // two tiles resident per unit (Q,dO or K,V)
constexpr uint32_t kOffRing = 2 * kTileBytes;
constexpr uint32_t kOffBar = kOffRing + kStages * kTileBytes;
constexpr uint32_t kOffVec = kOffBar + 256;      // per-block lse/Delta staging (dK/dV kernel)
constexpr uint32_t kSmemBytes = kOffVec + 2 * kBlk * 4 + 1024;

enum : uint32_t {
    kErrProducer = 1u << 0,
    kErrMma = 1u << 1,
    kErrElem = 1u << 2,
    kErrDrain = 1u << 3,
};

__device__ uint32_t g_fab_error_word;

struct Params {
    const void* o;        // forward output (dQ kernel: Delta)
    const float* lse;     // [BH, S_q] natural log
    float* delta;         // [BH, S_q]
    void* out0;           // dQ (dQ kernel) or dK (dK/dV kernel)
    void* out1;           // dV (dK/dV kernel)
    uint32_t S_q, S_k, BH, n_blk, num_pairs, causal;
    float scale, scale_log2;
};

struct Bars {
    uint64_t fixed_full, fixed_empty;
    uint64_t ring_full[kStages], ring_empty[kStages];
    uint64_t sdp_full, ds_full, acc_full;
    uint64_t mma_done;
};

// Work units (head, block), handed out as complementary pairs (b, n-1-b) of one head.
struct Units {
    uint32_t pi, second = 0;
    __device__ explicit Units(uint32_t first) : pi(first) {}
    __device__ __forceinline__ bool next(const Params& p, uint32_t& bh, uint32_t& blk) {
        const uint32_t per_head = (p.n_blk + 1) / 2;
        while (pi < p.num_pairs) {
            bh = pi / per_head;
            const uint32_t j = pi - bh * per_head;
            if (!second) {
                second = 1;
                blk = p.n_blk - 1 - j;
                return true;
            }
            second = 0;
            pi += gridDim.x;
            if (j != p.n_blk - 1 - j) {
                blk = j;
                return true;
            }
        }
        return false;
    }
};

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

template <bool kBF16>
__device__ __forceinline__ float2 unpack2(uint32_t w) {
    if (kBF16) return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

// D (M=128, N=128) = A (128 x 128, K-major smem) * B^T (128 x 128, K-major smem): 8 K-steps of 16.
__device__ __forceinline__ void issue_ss(uint32_t d_tmem, uint32_t a_addr, uint32_t b_addr, uint32_t idesc) {
    const Sw128Desc ad = make_sw128_desc2(a_addr, 16, 1024), bd = make_sw128_desc2(b_addr, 16, 1024);
#pragma unroll
    for (uint32_t kk = 0; kk < 8; ++kk) {
        const uint32_t off = ((kk >> 2) * kPanelBytes + (kk & 3) * 32) >> 4;
        mma_ss2(d_tmem, Sw128Desc{ad.lo + off, ad.hi}, Sw128Desc{bd.lo + off, bd.hi}, idesc, kk > 0);
    }
}

// D (M=128, N=128) (+)= A (128 x 128 16-bit in TMEM, K along columns) * B (128 K-rows x 128, MN-major smem).
__device__ __forceinline__ void issue_ts(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_addr, uint32_t idesc,
                                         bool accumulate) {
    const Sw128Desc bd = make_sw128_desc2(b_addr, kPanelBytes, 1024);
#pragma unroll
    for (uint32_t kk = 0; kk < 8; ++kk)
        mma_ts2(d_tmem, a_tmem + kk * 8, Sw128Desc{bd.lo + kk * (2048 >> 4), bd.hi}, idesc,
                (accumulate || kk > 0) ? 1u : 0u);
}

__device__ __forceinline__ uint32_t n_blocks(uint32_t S) { return (S + kBlk - 1) / kBlk; }

// Key blocks visible from query block qb (top-left causal: key k visible from row r when k <= r).
__device__ __forceinline__ uint32_t kv_blocks_for(const Params& p, uint32_t qb) {
    uint32_t nk = n_blocks(p.S_k);
    if (p.causal) {
        const uint32_t lim = qb + 1;
        if (lim < nk) nk = lim;
    }
    return nk;
}

// Query blocks [first, n) that see key block kb.
__device__ __forceinline__ uint32_t q_first_for(const Params& p, uint32_t kb) {
    return p.causal ? kb : 0u;
}

// 16-byte chunk c (8 elements) of row `row` of a 128-row tile stored as 64-column swizzle panels.
__device__ __forceinline__ uint4 tile_chunk(const uint8_t* tile, uint32_t row, uint32_t c) {
    return *reinterpret_cast<const uint4*>(tile + (c >> 3) * kPanelBytes + row * 128 + (((c & 7) ^ (row & 7)) << 4));
}

// Barrier among the 128 threads of the elementwise warpgroup only.
__device__ __forceinline__ void wg_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// The same barrier, returning the AND of `pred` over the warpgroup: every warp takes the same
// branch after it, so no warp can leave a loop that still has a barrier another warp waits on.
__device__ __forceinline__ bool wg_all(bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, 1, 128, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(pred))
        : "memory");
    return r != 0;
}

// ============================================================================================
// dQ (and Delta)
// ============================================================================================
template <bool kBF16>
__global__ void __launch_bounds__(kThreads, 1)
    fa_bwd_dq_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                     const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                     const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffBar + sizeof(Bars));
    volatile uint32_t* abort_flag = tmem_slot + 1;
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        mbar_init(&bars->fixed_full, 1);
        mbar_init(&bars->fixed_empty, 1);
        for (uint32_t s = 0; s < kStages; ++s) {
            mbar_init(&bars->ring_full[s], 1);
            mbar_init(&bars->ring_empty[s], 1);
        }
        mbar_init(&bars->sdp_full, 1);
        mbar_init(&bars->ds_full, 128);
        mbar_init(&bars->acc_full, 1);
        mbar_init(&bars->mma_done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 4) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const uint32_t sQ = smem_u32(smem + kOffFixed), sDO = sQ + kTileBytes, sRing = smem_u32(smem + kOffRing);
    // TMEM: S [0,128), dP [128,256), dQ [256,384); dS (16-bit) overlays S.
    if (warp == 5) {
        if (lane == 0) {
            uint32_t stage = 0, phase = 0, it = 0, pend_valid = 0, pend_phase = 0;
            int32_t fixed_pending = -1;
            bool ok = true;
            Units u(blockIdx.x);
            uint32_t bh, qb;
            for (; ok && u.next(p, bh, qb); ++it) {
                if (!mbar_wait_bounded(&bars->fixed_empty, (it & 1) ^ 1, abort_flag, &g_fab_error_word, kErrProducer)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&bars->fixed_full, 2 * kTileBytes);
                for (uint32_t h = 0; h < 2; ++h) {
                    tma_load_3d(smem + kOffFixed + h * kPanelBytes, &tm_q, &bars->fixed_full, h * 64, qb * kBlk, bh);
                    tma_load_3d(smem + kOffFixed + kTileBytes + h * kPanelBytes, &tm_do, &bars->fixed_full, h * 64,
                                qb * kBlk, bh);
                }
                fixed_pending = static_cast<int32_t>(it & 1);
                const uint32_t nkv = kv_blocks_for(p, qb);
                for (uint32_t j = 0; j < nkv && ok; ++j) {
                    for (uint32_t kv = 0; kv < 2; ++kv) {  // K_j, then V_j
                        if (!mbar_wait_bounded(&bars->ring_empty[stage], phase ^ 1, abort_flag, &g_fab_error_word,
                                               kErrProducer)) {
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(&bars->ring_full[stage], kTileBytes);
                        for (uint32_t h = 0; h < 2; ++h)
                            tma_load_3d(smem + kOffRing + stage * kTileBytes + h * kPanelBytes, kv ? &tm_v : &tm_k,
                                        &bars->ring_full[stage], h * 64, j * kBlk, bh);
                        pend_valid |= 1u << stage;
                        pend_phase = (pend_phase & ~(1u << stage)) | (phase << stage);
                        if (++stage == kStages) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                }
            }
            if (!ok) {
                volatile uint32_t never = 0;
                for (uint32_t s = 0; s < kStages; ++s)
                    if (pend_valid & (1u << s))
                        mbar_wait_bounded(&bars->ring_full[s], (pend_phase >> s) & 1u, &never, &g_fab_error_word,
                                          kErrDrain, 1000000000ull);
                if (fixed_pending >= 0)
                    mbar_wait_bounded(&bars->fixed_full, static_cast<uint32_t>(fixed_pending), &never,
                                      &g_fab_error_word, kErrDrain, 1000000000ull);
            }
        }
    } else if (warp == 4) {
        if (lane == 0) {
            const uint32_t idesc_ss = make_idesc_f16(kBF16, 128, 128, false, false);
            const uint32_t idesc_ts = make_idesc_f16(kBF16, 128, 128, false, true);
            const uint32_t tS = tmem_base, tDP = tmem_base + 128, tDQ = tmem_base + 256;
            uint32_t stage = 0, phase = 0, it = 0, ds_par = 0;
            bool ok = true;
            auto wait_ring = [&](uint32_t& st) -> bool {
                if (!mbar_wait_bounded(&bars->ring_full[stage], phase, abort_flag, &g_fab_error_word, kErrMma))
                    return false;
                tc_fence_after();
                st = stage;
                if (++stage == kStages) {
                    stage = 0;
                    phase ^= 1;
                }
                return true;
            };
            Units u(blockIdx.x);
            uint32_t bh, qb;
            for (; ok && u.next(p, bh, qb); ++it) {
                if (!mbar_wait_bounded(&bars->fixed_full, it & 1, abort_flag, &g_fab_error_word, kErrMma)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t nkv = kv_blocks_for(p, qb);
                for (uint32_t j = 0; j < nkv; ++j) {
                    uint32_t ks, vs;
                    if (!wait_ring(ks)) { ok = false; break; }
                    issue_ss(tS, sQ, sRing + ks * kTileBytes, idesc_ss);              // S = Q K_j^T
                    if (!wait_ring(vs)) { ok = false; break; }
                    issue_ss(tDP, sDO, sRing + vs * kTileBytes, idesc_ss);            // dP = dO V_j^T
                    tc_commit(&bars->sdp_full);
                    if (!mbar_wait_bounded(&bars->ds_full, ds_par, abort_flag, &g_fab_error_word, kErrMma)) {
                        ok = false;
                        break;
                    }
                    ds_par ^= 1;
                    tc_fence_after();
                    // Q and dO are free once the last dP is done and the elementwise warps, which
                    // read dO for Delta before their first dS, have arrived on ds_full.
                    if (j + 1 == nkv) tc_commit(&bars->fixed_empty);
                    issue_ts(tDQ, tS, sRing + ks * kTileBytes, idesc_ts, j > 0);      // dQ += dS K_j
                    tc_commit(&bars->ring_empty[ks]);
                    tc_commit(&bars->ring_empty[vs]);
                }
                if (!ok) break;
                tc_commit(&bars->acc_full);
            }
            tc_commit(&bars->mma_done);
            volatile uint32_t never = 0;
            mbar_wait_bounded(&bars->mma_done, 0, &never, &g_fab_error_word, kErrDrain, 1000000000ull);
        }
    } else {
        // ===================== elementwise: Delta, dS, dQ epilogue (row = thread) =====================
        const uint32_t t = threadIdx.x;  // TMEM lane = row within the block
        const uint32_t lane_field = ((warp & 3) * 32) << 16;
        const uint8_t* tDOs = smem + kOffFixed + kTileBytes;
        uint32_t it = 0, sdp_par = 0, acc_par = 0;
        Units u(blockIdx.x);
        uint32_t bh, qb;
        while (u.next(p, bh, qb)) {
            const uint32_t row = qb * kBlk + t;
            const bool valid = row < p.S_q;
            const size_t ridx = static_cast<size_t>(bh) * p.S_q + row;
            bool ok = mbar_wait_bounded(&bars->fixed_full, it & 1, abort_flag, &g_fab_error_word, kErrElem);
            if (!__all_sync(0xffffffffu, ok)) break;
            ++it;
            // Delta = rowsum(dO * O) for this row (dO from the staged tile, O from global).
            float delta = 0.f, lse2 = INFINITY;
            if (valid) {
                const uint4* orow = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.o) + ridx * 128);
#pragma unroll 4
                for (uint32_t c = 0; c < 16; ++c) {
                    const uint4 a = tile_chunk(tDOs, t, c), b = __ldg(orow + c);
                    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 x = unpack2<kBF16>(aw[e]), y = unpack2<kBF16>(bw[e]);
                        delta = fmaf(x.x, y.x, fmaf(x.y, y.y, delta));
                    }
                }
                p.delta[ridx] = delta;
                lse2 = p.lse[ridx] * 1.4426950408889634f;
            }
            const uint32_t nkv = kv_blocks_for(p, qb);
            for (uint32_t j = 0; j < nkv && ok; ++j) {
                ok = mbar_wait_bounded(&bars->sdp_full, sdp_par, abort_flag, &g_fab_error_word, kErrElem);
                if (!__all_sync(0xffffffffu, ok)) {
                    ok = false;
                    break;
                }
                sdp_par ^= 1;
                tc_fence_after();
                // keys of this block visible from this row: causal (k <= row) and the key tail
                int32_t lim = static_cast<int32_t>(p.S_k) - static_cast<int32_t>(j * kBlk);
                if (p.causal) {
                    const int32_t lc = static_cast<int32_t>(row) - static_cast<int32_t>(j * kBlk) + 1;
                    if (lc < lim) lim = lc;
                }
#pragma unroll 1
                for (int c = 0; c < 4; ++c) {
                    uint32_t s[32], dp[32], pk[16];
                    tmem_ld32(tmem_base + c * 32 + lane_field, s);
                    tmem_ld32(tmem_base + 128 + c * 32 + lane_field, dp);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        float ds[2];
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const int key = c * 32 + 2 * e + h;
                            const float pr = key < lim ? ex2(__uint_as_float(s[2 * e + h]) * p.scale_log2 - lse2) : 0.f;
                            ds[h] = pr * (__uint_as_float(dp[2 * e + h]) - delta);
                        }
                        pk[e] = pack2<kBF16>(ds[0], ds[1]);
                    }
                    tmem_st16(tmem_base + c * 16 + lane_field, pk);
                }
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(&bars->ds_full);
            }
            if (!ok) break;
            ok = mbar_wait_bounded(&bars->acc_full, acc_par, abort_flag, &g_fab_error_word, kErrElem);
            if (!__all_sync(0xffffffffu, ok)) break;
            acc_par ^= 1;
            tc_fence_after();
            uint8_t* dq_row = static_cast<uint8_t*>(p.out0) + ridx * 128 * 2;
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
                uint32_t acc[32], pk[16];
                tmem_ld32(tmem_base + 256 + c * 32 + lane_field, acc);
                tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 16; ++e)
                    pk[e] = pack2<kBF16>(__uint_as_float(acc[2 * e]) * p.scale, __uint_as_float(acc[2 * e + 1]) * p.scale);
                if (valid) {
                    uint4* dst = reinterpret_cast<uint4*>(dq_row + c * 64);
#pragma unroll
                    for (int v = 0; v < 4; ++v) dst[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
                }
            }
            tc_fence_before();
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 4) {
        __syncwarp();
        tmem_dealloc(tmem_base, 512);
    }
}

// ============================================================================================
// dK, dV
// ============================================================================================
template <bool kBF16>
__global__ void __launch_bounds__(kThreads, 1)
    fa_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                       const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                       const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffBar + sizeof(Bars));
    volatile uint32_t* abort_flag = tmem_slot + 1;
    float* s_lse = reinterpret_cast<float*>(smem + kOffVec);
    float* s_delta = s_lse + kBlk;
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const uint32_t nq = n_blocks(p.S_q);
    if (threadIdx.x == 0) {
        mbar_init(&bars->fixed_full, 1);
        mbar_init(&bars->fixed_empty, 1);
        for (uint32_t s = 0; s < kStages; ++s) {
            mbar_init(&bars->ring_full[s], 1);
            mbar_init(&bars->ring_empty[s], 1);
        }
        mbar_init(&bars->sdp_full, 1);
        mbar_init(&bars->ds_full, 128);
        mbar_init(&bars->acc_full, 1);
        mbar_init(&bars->mma_done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 4) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const uint32_t sK = smem_u32(smem + kOffFixed), sV = sK + kTileBytes, sRing = smem_u32(smem + kOffRing);
    // TMEM: S^T [0,128), dP^T [128,256), dV [256,384), dK [384,512); P^T over S^T, dS^T over dP^T.
    if (warp == 5) {
        if (lane == 0) {
            uint32_t stage = 0, phase = 0, it = 0, pend_valid = 0, pend_phase = 0;
            int32_t fixed_pending = -1;
            bool ok = true;
            Units u(blockIdx.x);
            uint32_t bh, kb;
            while (ok && u.next(p, bh, kb)) {
                const uint32_t q0 = q_first_for(p, kb);
                if (q0 >= nq) continue;  // no query sees these keys: the MMA and epilogue skip the unit too
                if (!mbar_wait_bounded(&bars->fixed_empty, (it & 1) ^ 1, abort_flag, &g_fab_error_word, kErrProducer)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&bars->fixed_full, 2 * kTileBytes);
                for (uint32_t h = 0; h < 2; ++h) {
                    tma_load_3d(smem + kOffFixed + h * kPanelBytes, &tm_k, &bars->fixed_full, h * 64, kb * kBlk, bh);
                    tma_load_3d(smem + kOffFixed + kTileBytes + h * kPanelBytes, &tm_v, &bars->fixed_full, h * 64,
                                kb * kBlk, bh);
                }
                fixed_pending = static_cast<int32_t>(it & 1);
                ++it;
                for (uint32_t i = q0; i < nq && ok; ++i) {
                    for (uint32_t x = 0; x < 2; ++x) {  // Q_i, then dO_i
                        if (!mbar_wait_bounded(&bars->ring_empty[stage], phase ^ 1, abort_flag, &g_fab_error_word,
                                               kErrProducer)) {
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(&bars->ring_full[stage], kTileBytes);
                        for (uint32_t h = 0; h < 2; ++h)
                            tma_load_3d(smem + kOffRing + stage * kTileBytes + h * kPanelBytes, x ? &tm_do : &tm_q,
                                        &bars->ring_full[stage], h * 64, i * kBlk, bh);
                        pend_valid |= 1u << stage;
                        pend_phase = (pend_phase & ~(1u << stage)) | (phase << stage);
                        if (++stage == kStages) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                }
            }
            if (!ok) {
                volatile uint32_t never = 0;
                for (uint32_t s = 0; s < kStages; ++s)
                    if (pend_valid & (1u << s))
                        mbar_wait_bounded(&bars->ring_full[s], (pend_phase >> s) & 1u, &never, &g_fab_error_word,
                                          kErrDrain, 1000000000ull);
                if (fixed_pending >= 0)
                    mbar_wait_bounded(&bars->fixed_full, static_cast<uint32_t>(fixed_pending), &never,
                                      &g_fab_error_word, kErrDrain, 1000000000ull);
            }
        }
    } else if (warp == 4) {
        if (lane == 0) {
            const uint32_t idesc_ss = make_idesc_f16(kBF16, 128, 128, false, false);
            const uint32_t idesc_ts = make_idesc_f16(kBF16, 128, 128, false, true);
            const uint32_t tS = tmem_base, tDP = tmem_base + 128, tDV = tmem_base + 256, tDK = tmem_base + 384;
            uint32_t stage = 0, phase = 0, it = 0, ds_par = 0;
            bool ok = true;
            auto wait_ring = [&](uint32_t& st) -> bool {
                if (!mbar_wait_bounded(&bars->ring_full[stage], phase, abort_flag, &g_fab_error_word, kErrMma))
                    return false;
                tc_fence_after();
                st = stage;
                if (++stage == kStages) {
                    stage = 0;
                    phase ^= 1;
                }
                return true;
            };
            Units u(blockIdx.x);
            uint32_t bh, kb;
            while (ok && u.next(p, bh, kb)) {
                const uint32_t q0 = q_first_for(p, kb);
                if (q0 >= nq) continue;  // the producer skipped this unit too
                if (!mbar_wait_bounded(&bars->fixed_full, it & 1, abort_flag, &g_fab_error_word, kErrMma)) {
                    ok = false;
                    break;
                }
                ++it;
                tc_fence_after();
                for (uint32_t i = q0; i < nq; ++i) {
                    uint32_t qs, os;
                    if (!wait_ring(qs)) { ok = false; break; }
                    issue_ss(tS, sK, sRing + qs * kTileBytes, idesc_ss);              // S^T = K Q_i^T
                    if (!wait_ring(os)) { ok = false; break; }
                    issue_ss(tDP, sV, sRing + os * kTileBytes, idesc_ss);             // dP^T = V dO_i^T
                    tc_commit(&bars->sdp_full);
                    if (!mbar_wait_bounded(&bars->ds_full, ds_par, abort_flag, &g_fab_error_word, kErrMma)) {
                        ok = false;
                        break;
                    }
                    ds_par ^= 1;
                    tc_fence_after();
                    issue_ts(tDV, tS, sRing + os * kTileBytes, idesc_ts, i > q0);     // dV += P^T dO_i
                    issue_ts(tDK, tDP, sRing + qs * kTileBytes, idesc_ts, i > q0);    // dK += dS^T Q_i
                    tc_commit(&bars->ring_empty[qs]);
                    tc_commit(&bars->ring_empty[os]);
                }
                if (!ok) break;
                tc_commit(&bars->fixed_empty);
                tc_commit(&bars->acc_full);
            }
            tc_commit(&bars->mma_done);
            volatile uint32_t never = 0;
            mbar_wait_bounded(&bars->mma_done, 0, &never, &g_fab_error_word, kErrDrain, 1000000000ull);
        }
    } else {
        // =================== elementwise: P^T, dS^T, dK/dV epilogue (key = thread) ===================
        const uint32_t t = threadIdx.x;  // TMEM lane = key within the block
        const uint32_t lane_field = ((warp & 3) * 32) << 16;
        uint32_t sdp_par = 0, acc_par = 0;
        Units u(blockIdx.x);
        uint32_t bh, kb;
        bool ok = true;
        while (ok && u.next(p, bh, kb)) {
            const uint32_t key = kb * kBlk + t;
            const size_t kidx = static_cast<size_t>(bh) * p.S_k + key;
            const uint32_t q0 = q_first_for(p, kb);
            if (q0 < nq) {
                for (uint32_t i = q0; i < nq; ++i) {
                    // stage lse (log2 domain; +inf for rows past S_q, so their P is 0) and Delta of block i
                    wg_sync();  // every thread is done reading the previous block's values
                    const uint32_t r = i * kBlk + t;
                    const size_t ridx = static_cast<size_t>(bh) * p.S_q + r;
                    s_lse[t] = r < p.S_q ? p.lse[ridx] * 1.4426950408889634f : INFINITY;
                    s_delta[t] = r < p.S_q ? p.delta[ridx] : 0.f;
                    // publishes the staged values and makes the give-up decision uniform
                    ok = wg_all(mbar_wait_bounded(&bars->sdp_full, sdp_par, abort_flag, &g_fab_error_word, kErrElem));
                    if (!ok) break;
                    sdp_par ^= 1;
                    tc_fence_after();
                    // rows of block i that see this key: causal (key <= row), i.e. row index >= first
                    const int32_t first = p.causal ? static_cast<int32_t>(key) - static_cast<int32_t>(i * kBlk) : 0;
#pragma unroll 1
                    for (int c = 0; c < 4; ++c) {
                        uint32_t s[32], dp[32], pp[16], pd[16];
                        tmem_ld32(tmem_base + c * 32 + lane_field, s);
                        tmem_ld32(tmem_base + 128 + c * 32 + lane_field, dp);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 16; ++e) {
                            float pr[2], ds[2];
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                const int col = c * 32 + 2 * e + h;
                                pr[h] = col >= first ? ex2(__uint_as_float(s[2 * e + h]) * p.scale_log2 - s_lse[col]) : 0.f;
                                ds[h] = pr[h] * (__uint_as_float(dp[2 * e + h]) - s_delta[col]);
                            }
                            pp[e] = pack2<kBF16>(pr[0], pr[1]);
                            pd[e] = pack2<kBF16>(ds[0], ds[1]);
                        }
                        tmem_st16(tmem_base + c * 16 + lane_field, pp);
                        tmem_st16(tmem_base + 128 + c * 16 + lane_field, pd);
                    }
                    tmem_wait_st();
                    tc_fence_before();
                    mbar_arrive(&bars->ds_full);
                }
                if (!ok) break;
                ok = wg_all(mbar_wait_bounded(&bars->acc_full, acc_par, abort_flag, &g_fab_error_word, kErrElem));
                if (!ok) break;
                acc_par ^= 1;
                tc_fence_after();
            }
            // epilogue: dV, dK (scaled) of this key; zeros when no query sees the block
            const bool valid = key < p.S_k;
            uint8_t* dk_row = static_cast<uint8_t*>(p.out0) + kidx * 128 * 2;
            uint8_t* dv_row = static_cast<uint8_t*>(p.out1) + kidx * 128 * 2;
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
                uint32_t av[32], ak[32], pv[16], pk[16];
                if (q0 < nq) {
                    tmem_ld32(tmem_base + 256 + c * 32 + lane_field, av);
                    tmem_ld32(tmem_base + 384 + c * 32 + lane_field, ak);
                    tmem_wait_ld();
                } else {
#pragma unroll
                    for (int e = 0; e < 32; ++e) av[e] = ak[e] = 0u;
                }
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    pv[e] = pack2<kBF16>(__uint_as_float(av[2 * e]), __uint_as_float(av[2 * e + 1]));
                    pk[e] = pack2<kBF16>(__uint_as_float(ak[2 * e]) * p.scale, __uint_as_float(ak[2 * e + 1]) * p.scale);
                }
                if (valid) {
                    uint4* dv = reinterpret_cast<uint4*>(dv_row + c * 64);
                    uint4* dk = reinterpret_cast<uint4*>(dk_row + c * 64);
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        dv[v] = make_uint4(pv[4 * v], pv[4 * v + 1], pv[4 * v + 2], pv[4 * v + 3]);
                        dk[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
                    }
                }
            }
            tc_fence_before();
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 4) {
        __syncwarp();
        tmem_dealloc(tmem_base, 512);
    }
}

// ============================================================================================
// SIMT path (fp32 math): Delta + dQ with a warp per query row, dK/dV with a warp per key row.
// ============================================================================================
template <typename T>
__global__ void __launch_bounds__(256) fa_bwd_simt_dq_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                             const T* __restrict__ v, const T* __restrict__ o,
                                                             const T* __restrict__ dO, const float* __restrict__ lse,
                                                             float* __restrict__ delta, T* __restrict__ dq,
                                                             uint32_t BH, uint32_t S_q, uint32_t S_k, uint32_t D,
                                                             uint32_t Dv, float scale, uint32_t causal) {
    constexpr int kMaxD = 256;
    __shared__ float qs[8][kMaxD], dos[8][kMaxD];
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const uint64_t rows = static_cast<uint64_t>(BH) * S_q;
    for (uint64_t gr = static_cast<uint64_t>(blockIdx.x) * 8 + warp; gr < rows; gr += static_cast<uint64_t>(gridDim.x) * 8) {
        const uint64_t bh = gr / S_q;
        const uint32_t qi = static_cast<uint32_t>(gr % S_q);
        float dl = 0.f;
        for (uint32_t d = lane; d < D; d += 32) qs[warp][d] = elem<T>::to_f(q[gr * D + d]);
        for (uint32_t d = lane; d < Dv; d += 32) {
            const float g = elem<T>::to_f(dO[gr * Dv + d]);
            dos[warp][d] = g;
            dl = fmaf(g, elem<T>::to_f(o[gr * Dv + d]), dl);
        }
        dl = warp_sum(dl);
        if (lane == 0) delta[gr] = dl;
        __syncwarp();
        const float l = lse[gr];
        float acc[kMaxD / 32];
#pragma unroll
        for (int i = 0; i < kMaxD / 32; ++i) acc[i] = 0.f;
        const uint32_t kend = causal ? min(S_k, qi + 1) : S_k;
        for (uint32_t k0 = 0; k0 < kend; k0 += 32) {
            const uint32_t kj = k0 + lane;
            float ds = 0.f;
            if (kj < kend) {
                const T* krow = k + (bh * S_k + kj) * D;
                const T* vrow = v + (bh * S_k + kj) * Dv;
                float s = 0.f, dp = 0.f;
                for (uint32_t d = 0; d < D; ++d) s = fmaf(qs[warp][d], elem<T>::to_f(krow[d]), s);
                for (uint32_t d = 0; d < Dv; ++d) dp = fmaf(dos[warp][d], elem<T>::to_f(vrow[d]), dp);
                const float pr = expf(s * scale - l);
                ds = pr * (dp - dl);
            }
            const uint32_t cnt = min(32u, kend - k0);
            for (uint32_t jj = 0; jj < cnt; ++jj) {
                const float g = __shfl_sync(0xffffffffu, ds, jj);
                const T* krow = k + (bh * S_k + k0 + jj) * D;
#pragma unroll
                for (int i = 0; i < kMaxD / 32; ++i) {
                    const uint32_t d = lane + 32 * i;
                    if (d < D) acc[i] = fmaf(g, elem<T>::to_f(krow[d]), acc[i]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < kMaxD / 32; ++i) {
            const uint32_t d = lane + 32 * i;
            if (d < D) dq[gr * D + d] = elem<T>::from_f(acc[i] * scale);
        }
        __syncwarp();
    }
}

template <typename T>
__global__ void __launch_bounds__(256) fa_bwd_simt_dkdv_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                               const T* __restrict__ v, const T* __restrict__ dO,
                                                               const float* __restrict__ lse,
                                                               const float* __restrict__ delta, T* __restrict__ dk,
                                                               T* __restrict__ dv, uint32_t BH, uint32_t S_q,
                                                               uint32_t S_k, uint32_t D, uint32_t Dv, float scale,
                                                               uint32_t causal) {
    constexpr int kMaxD = 256;
    __shared__ float ks[8][kMaxD], vs[8][kMaxD];
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const uint64_t keys = static_cast<uint64_t>(BH) * S_k;
    for (uint64_t gk = static_cast<uint64_t>(blockIdx.x) * 8 + warp; gk < keys; gk += static_cast<uint64_t>(gridDim.x) * 8) {
        const uint64_t bh = gk / S_k;
        const uint32_t kj = static_cast<uint32_t>(gk % S_k);
        for (uint32_t d = lane; d < D; d += 32) ks[warp][d] = elem<T>::to_f(k[gk * D + d]);
        for (uint32_t d = lane; d < Dv; d += 32) vs[warp][d] = elem<T>::to_f(v[gk * Dv + d]);
        __syncwarp();
        float ak[kMaxD / 32], av[kMaxD / 32];
#pragma unroll
        for (int i = 0; i < kMaxD / 32; ++i) ak[i] = av[i] = 0.f;
        const uint32_t r_begin = causal ? kj : 0u;
        for (uint32_t r0 = r_begin; r0 < S_q; r0 += 32) {
            const uint32_t r = r0 + lane;
            float pr = 0.f, ds = 0.f;
            if (r < S_q) {
                const T* qrow = q + (bh * S_q + r) * D;
                const T* drow = dO + (bh * S_q + r) * Dv;
                float s = 0.f, dp = 0.f;
                for (uint32_t d = 0; d < D; ++d) s = fmaf(elem<T>::to_f(qrow[d]), ks[warp][d], s);
                for (uint32_t d = 0; d < Dv; ++d) dp = fmaf(elem<T>::to_f(drow[d]), vs[warp][d], dp);
                pr = expf(s * scale - lse[bh * S_q + r]);
                ds = pr * (dp - delta[bh * S_q + r]);
            }
            const uint32_t cnt = min(32u, S_q - r0);
            for (uint32_t jj = 0; jj < cnt; ++jj) {
                const float gp = __shfl_sync(0xffffffffu, pr, jj), gs = __shfl_sync(0xffffffffu, ds, jj);
                const T* qrow = q + (bh * S_q + r0 + jj) * D;
                const T* drow = dO + (bh * S_q + r0 + jj) * Dv;
#pragma unroll
                for (int i = 0; i < kMaxD / 32; ++i) {
                    const uint32_t d = lane + 32 * i;
                    if (d < D) ak[i] = fmaf(gs, elem<T>::to_f(qrow[d]), ak[i]);
                    if (d < Dv) av[i] = fmaf(gp, elem<T>::to_f(drow[d]), av[i]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < kMaxD / 32; ++i) {
            const uint32_t d = lane + 32 * i;
            if (d < D) dk[gk * D + d] = elem<T>::from_f(ak[i] * scale);
            if (d < Dv) dv[gk * Dv + d] = elem<T>::from_f(av[i]);
        }
        __syncwarp();
    }
}

uint32_t read_error_word(const char** name) {
    *name = "flash_attention_bwd";
    uint32_t word = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&word, g_fab_error_word, sizeof(word)) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (word) cudaMemcpyToSymbol(g_fab_error_word, &zero, sizeof(zero));
    return word;
}

thread_local int t_last_path = 0;

template <bool kBF16>
int launch_tc(const void* q, const void* k, const void* v, const void* o, const void* dO, const float* lse, void* dq,
              void* dk, void* dv, float* delta, const flash_attention_fwd_fused_tiling_data* t, cudaStream_t stream) {
    static std::once_flag reg_once;
    std::call_once(reg_once, [] { register_error_word(read_error_word); });
    const uint64_t BH = static_cast<uint64_t>(t->B) * t->H;
    const CUtensorMapDataType dt = kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const uint32_t box[3] = {64, 128, 1};
    CUtensorMap tmq, tmdo, tmk, tmv;
    {
        uint64_t dims[3] = {128, t->S_q, BH};
        uint64_t strides[2] = {256, static_cast<uint64_t>(t->S_q) * 256};
        if (int rc = encode_tmap(&tmq, dt, 3, q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
        if (int rc = encode_tmap(&tmdo, dt, 3, dO, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
    }
    {
        uint64_t dims[3] = {128, t->S_k, BH};
        uint64_t strides[2] = {256, static_cast<uint64_t>(t->S_k) * 256};
        if (int rc = encode_tmap(&tmk, dt, 3, k, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
        if (int rc = encode_tmap(&tmv, dt, 3, v, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
    }
    if (BH * ((t->S_q + kBlk - 1) / kBlk + (t->S_k + kBlk - 1) / kBlk) > 0xffffffffull)
        return fail(HC_ERR_UNSUPPORTED, "flash_attention_bwd: too many work units");
    Params prm;
    prm.o = o;
    prm.lse = lse;
    prm.delta = delta;
    prm.S_q = t->S_q;
    prm.S_k = t->S_k;
    prm.BH = static_cast<uint32_t>(BH);
    prm.causal = t->maskType;
    prm.scale = t->scale;
    prm.scale_log2 = t->scale * 1.4426950408889634f;
    for (int pass = 0; pass < 2; ++pass) {  // dQ (and Delta) first: the dK/dV kernel reads Delta
        const void* fn = pass == 0 ? reinterpret_cast<const void*>(fa_bwd_dq_kernel<kBF16>)
                                   : reinterpret_cast<const void*>(fa_bwd_dkdv_kernel<kBF16>);
        if (int rc = set_max_dynamic_smem(fn, kSmemBytes, pass == 0 ? "fa_bwd_dq_kernel" : "fa_bwd_dkdv_kernel"))
            return rc;
        prm.n_blk = pass == 0 ? (t->S_q + kBlk - 1) / kBlk : (t->S_k + kBlk - 1) / kBlk;
        prm.num_pairs = static_cast<uint32_t>(BH * ((prm.n_blk + 1) / 2));
        prm.out0 = pass == 0 ? dq : dk;
        prm.out1 = dv;
        uint32_t grid = static_cast<uint32_t>(sm_count());
        if (grid > prm.num_pairs) grid = prm.num_pairs;
        if (pass == 0)
            fa_bwd_dq_kernel<kBF16><<<grid, kThreads, kSmemBytes, stream>>>(tmq, tmdo, tmk, tmv, prm);
        else
            fa_bwd_dkdv_kernel<kBF16><<<grid, kThreads, kSmemBytes, stream>>>(tmq, tmdo, tmk, tmv, prm);
        if (int rc = check_launch(pass == 0 ? "fa_bwd_dq_kernel" : "fa_bwd_dkdv_kernel")) return rc;
    }
    t_last_path = 1;
    return HC_OK;
}

template <typename T>
int launch_simt(const void* q, const void* k, const void* v, const void* o, const void* dO, const float* lse, void* dq,
                void* dk, void* dv, float* delta, const flash_attention_fwd_fused_tiling_data* t, cudaStream_t stream) {
    const uint32_t BH = t->B * t->H;
    const uint64_t cap_q = static_cast<uint64_t>(resident_blocks(reinterpret_cast<const void*>(fa_bwd_simt_dq_kernel<T>), 256, 0));
    const uint64_t cap_k = static_cast<uint64_t>(resident_blocks(reinterpret_cast<const void*>(fa_bwd_simt_dkdv_kernel<T>), 256, 0));
    uint64_t bq = (static_cast<uint64_t>(BH) * t->S_q + 7) / 8, bk = (static_cast<uint64_t>(BH) * t->S_k + 7) / 8;
    if (bq > cap_q) bq = cap_q;
    if (bk > cap_k) bk = cap_k;
    fa_bwd_simt_dq_kernel<T><<<static_cast<unsigned>(bq), 256, 0, stream>>>(
        static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(v), static_cast<const T*>(o),
        static_cast<const T*>(dO), lse, delta, static_cast<T*>(dq), BH, t->S_q, t->S_k, t->D, t->D_v, t->scale,
        t->maskType);
    if (int rc = check_launch("fa_bwd_simt_dq_kernel")) return rc;
    fa_bwd_simt_dkdv_kernel<T><<<static_cast<unsigned>(bk), 256, 0, stream>>>(
        static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(v), static_cast<const T*>(dO), lse,
        delta, static_cast<T*>(dk), static_cast<T*>(dv), BH, t->S_q, t->S_k, t->D, t->D_v, t->scale, t->maskType);
    if (int rc = check_launch("fa_bwd_simt_dkdv_kernel")) return rc;
    t_last_path = 2;
    return HC_OK;
}

}  // namespace fab
}  // namespace hc

using namespace hc;

extern "C" int hc_flash_attention_bwd_launch(const void* q, const void* k, const void* v, const void* o,
                                             const void* dO, const float* lse, void* dq, void* dk, void* dv,
                                             float* delta, const flash_attention_fwd_fused_tiling_data* t, int dtype,
                                             void* stream) {
    if (int rc = fa_check_tiling(t, t ? t->H : 1u, dtype)) return rc;
    if (t->B == 0 || t->H == 0 || t->S_q == 0) return ok();
    if (!q || !k || !v || !o || !dO || !lse || !dq || !dk || !dv || !delta)
        return fail(HC_ERR_INVALID, "flash_attention_bwd: null pointer");
    if (fault_hit("launch")) return fail(HC_ERR_INJECTED, "flash_attention_bwd: injected launch failure");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool tc_shape = t->D == 128 && t->D_v == 128 && t->scale > 0.f && aligned16(q) && aligned16(k) &&
                          aligned16(v) && aligned16(o) && aligned16(dO) && aligned16(dq) && aligned16(dk) &&
                          aligned16(dv);
    if (dtype == HC_DTYPE_BF16)
        return tc_shape ? fab::launch_tc<true>(q, k, v, o, dO, lse, dq, dk, dv, delta, t, s)
                        : fab::launch_simt<bf16_t>(q, k, v, o, dO, lse, dq, dk, dv, delta, t, s);
    if (dtype == HC_DTYPE_F16)
        return tc_shape ? fab::launch_tc<false>(q, k, v, o, dO, lse, dq, dk, dv, delta, t, s)
                        : fab::launch_simt<f16_t>(q, k, v, o, dO, lse, dq, dk, dv, delta, t, s);
    return fab::launch_simt<float>(q, k, v, o, dO, lse, dq, dk, dv, delta, t, s);
}

extern "C" int hc_flash_attention_bwd_last_path(void) { return fab::t_last_path; }
