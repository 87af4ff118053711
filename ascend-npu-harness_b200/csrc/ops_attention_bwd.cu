// flash_attention backward on B200: dQ, dK, dV of O = softmax(Q K^T * scale [+ causal mask]) V
// from Q, K, V, O, dO and the forward's lse (natural log).  The harness has no backward (its
// ladder is forward only); the math is the standard one:
//   P = exp(S * scale - lse), dV = P^T dO, dP = dO V^T, Delta = rowsum(dO * O),
//   dS = P * (dP - Delta), dQ = scale * dS K, dK = scale * dS^T Q.
//
// Tensor-core path (bf16/fp16, D = D_v = 64 or 128, 16-byte aligned buffers): two kernels with the same
// structure.  A CTA holds two 128 x D "fixed" tiles of one 128-row block in shared memory and
// streams the other side's 128-row tiles through a 5-stage TMA ring.  Each streamed tile is released
// as soon as its last product is issued (V_j and dO_i after one product, K_j and Q_i after two), and
// the MMA warp waits for each tile just before its first product, so loads run about a block ahead:
//   * fa_bwd_dq_kernel: fixed Q, dO of a query block (rows on TMEM lanes); for every visible key
//     block j: S = Q K_j^T, dP = dO V_j^T, dS = P (dP - Delta) (16-bit), dQ += dS K_j.  It first
//     computes Delta = rowsum(dO * O) for its rows and writes it (the caller's [B, H, S_q] fp32
//     buffer).  TMEM: S [0,128), dP in two buffers [128,256) and [256,384) (block j in buffer j & 1,
//     dS packed over it), dQ from column 384 (D columns).
//   * fa_bwd_dkdv_kernel (launched after, it reads Delta): fixed K, V of a key block (keys on
//     TMEM lanes); for every query block i that sees the keys: S^T = K Q_i^T, dP^T = V dO_i^T,
//     P^T (16-bit, over S^T), dS^T (16-bit, over dP^T), dV += P^T dO_i, dK += dS^T Q_i.
//     TMEM: S^T [0,128), dP^T [128,256), dV from column 256, dK from column 384 (D columns each).
// Every product is M=128, K=16 per instruction, N=128 for S and dP and N=D for dQ, dK, dV: at D=128
// one tcgen05.mma every 64 cycles at the full tensor rate (an SS product with N = 64 runs at two thirds
// of it, bound by shared-memory operand reads).  The kWG
// elementwise warpgroups (warps 4g..4g+3; a thread owns one TMEM lane, warpgroup g the kCols columns
// [kCols*g, kCols*(g+1)) of each tile) work in two phases per block, each with its own hand-off to
// the MMA warp (warp 4*kWG), which keeps the tensor pipe busy during both:
//   dQ:    phase 1 loads S and releases it (the next S is issued at once), forms P in registers;
//          phase 2 forms dS from dP and packs it over dP (ds_full): dQ += dS K_j, then dP of block
//          j + 2 into the same buffer, so phase 2 of the next block never waits for this product.
//   dK/dV: phase 1 forms P^T from S^T and packs it over S^T (p_full): dV += P^T dO_i, then the next
//          S^T; phase 2 forms dS^T and packs it over dP^T (ds_full): dK += dS^T Q_i, then the next
//          dP^T.
// The accumulators of the next work unit are started only after every warpgroup's epilogue has
// read them (acc_empty).  Warp 4*kWG+1 issues TMA (no multicast).  The causal mask is applied only on the
// diagonal block; tails need none (rows past S_q get lse = +inf, so P = 0; keys past S_k meet zero
// K/V rows or land in accumulator rows that are not stored).  Work units are handed out as
// complementary block pairs (b, n-1-b) of one head so that every CTA gets the same causal work.
// Every mbarrier wait is bounded as in the forward kernel, and the threads of a warpgroup take
// each give-up decision together (a barrier that ANDs their results), so none is left at a barrier.
//
// SIMT path: fp32, or any other head dims (<= 256): a warp per query row for dQ/Delta and a
// warp per key row for dK/dV, fp32 math.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <mutex>
#include <type_traits>

#include "hc_device.cuh"
#include "hc_internal.h"
#include "sm100.cuh"
#include "tmap.h"

namespace hc {
namespace fab {

using namespace sm100;

constexpr uint32_t kBlk = 128;                  // rows (queries or keys) per block
constexpr uint32_t kPanelBytes = 128 * 64 * 2;  // one 64-column swizzle panel of a 128-row tile: 16 KB
constexpr uint32_t kWG = 2;                     // elementwise warpgroups
constexpr uint32_t kCols = kBlk / kWG;          // columns of a tile per warpgroup
constexpr uint32_t kChunks = kCols / 32;        // 32-column TMEM loads per thread and tile
constexpr uint32_t kStepsWG = kCols / 16;       // K-steps of a TMEM-operand product per warpgroup
constexpr uint32_t kElem = 128 * kWG;           // elementwise threads
constexpr uint32_t kMmaWarp = 4 * kWG, kTmaWarp = 4 * kWG + 1;
constexpr uint32_t kThreads = kElem + 64;       // elementwise warpgroups, the MMA warp, the TMA warp
constexpr uint32_t kStages = 5;                 // streamed-tile ring (tiles are released one by one)
constexpr uint32_t kOffFixed = 0;               // two tiles resident per unit (Q,dO or K,V)
constexpr uint32_t kVecBytes = kWG * 2 * kCols * 4;

// Shared-memory layout and epilogue split for head dim HD (64 or 128; D = D_v): a 128-row tile is
// HD/64 swizzle panels; the ring follows the two fixed tiles; dQ / dK / dV rows are written
// kOutCols columns per warpgroup.
template <uint32_t HD>
struct Dims {
    static_assert(HD == 64 || HD == 128, "head dims 64 and 128");
    static constexpr uint32_t kPanels = HD / 64;
    static constexpr uint32_t kTileBytes = kPanels * kPanelBytes;
    static constexpr uint32_t kOffRing = 2 * kTileBytes;
    static constexpr uint32_t kOffBar = kOffRing + kStages * kTileBytes;
    static constexpr uint32_t kOffVec = kOffBar + 256;  // dK/dV: per warpgroup, -lse*log2(e) and Delta of its kCols queries
    static constexpr uint32_t kSmemBytes = kOffVec + kVecBytes + 1024;
    static constexpr uint32_t kOutCols = HD / kWG;
    static constexpr uint32_t kOutChunks = kOutCols / 32;
    static_assert(kOutCols % 32 == 0, "32-column TMEM loads per warpgroup");
};

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
    uint64_t s_full, dp_full[2];   // MMA -> elementwise: S (S^T) and dP (dP^T, buffer b) of the block are in TMEM
    uint64_t mid, ds_full;         // elementwise -> MMA (kElem arrivals): phase 1 done (dQ: S read; dK/dV: P^T packed), phase 2 (dS packed)
    uint64_t acc_full, acc_empty;
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

// Barrier among the 128 threads of warpgroup g (named barrier 2 + g), returning the AND of `pred`
// over them: the warpgroup takes the same branch after it, so no warp can leave a loop that still
// has a barrier another warp of the group waits on.
__device__ __forceinline__ bool wg_all(uint32_t g, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, %2, 128, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(pred)), "r"(2 + g)
        : "memory");
    return r != 0;
}

// Plain barrier among the 128 threads of warpgroup g.
__device__ __forceinline__ void wg_sync(uint32_t g) { asm volatile("bar.sync %0, 128;" ::"r"(2 + g) : "memory"); }

// Shared setup of both kernels: barriers, TMEM (512 columns, MMA warp), and the bounded-wait state.
__device__ __forceinline__ uint32_t setup_cta(Bars* bars, uint32_t* tmem_slot, volatile uint32_t* abort_flag,
                                              uint32_t warp) {
    if (threadIdx.x == 0) {
        mbar_init(&bars->fixed_full, 1);
        mbar_init(&bars->fixed_empty, 1);
        for (uint32_t s = 0; s < kStages; ++s) {
            mbar_init(&bars->ring_full[s], 1);
            mbar_init(&bars->ring_empty[s], 1);
        }
        mbar_init(&bars->s_full, 1);
        mbar_init(&bars->dp_full[0], 1);
        mbar_init(&bars->dp_full[1], 1);
        mbar_init(&bars->mid, kElem);
        mbar_init(&bars->ds_full, kElem);
        mbar_init(&bars->acc_full, 1);
        mbar_init(&bars->acc_empty, kElem);
        mbar_init(&bars->mma_done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    return *tmem_slot;
}

__device__ __forceinline__ void teardown_cta(uint32_t tmem_base, uint32_t warp) {
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kMmaWarp) {
        __syncwarp();
        tmem_dealloc(tmem_base, 512);
    }
}

// The producer's wait for a free ring slot, its loads, and the drain after a give-up: every
// issued load is waited for (bounded) so no copy lands in shared memory after the CTA exits.
struct Ring {
    uint32_t stage = 0, phase = 0, pend_valid = 0, pend_phase = 0;
    template <uint32_t HD>
    __device__ __forceinline__ bool load(Bars* bars, uint8_t* smem, const CUtensorMap* tm, uint32_t row_blk,
                                         uint32_t bh, volatile uint32_t* abort_flag) {
        using D = Dims<HD>;
        if (!mbar_wait_bounded(&bars->ring_empty[stage], phase ^ 1, abort_flag, &g_fab_error_word, kErrProducer))
            return false;
        mbar_arrive_expect_tx(&bars->ring_full[stage], D::kTileBytes);
        for (uint32_t h = 0; h < D::kPanels; ++h)
            tma_load_3d(smem + D::kOffRing + stage * D::kTileBytes + h * kPanelBytes, tm, &bars->ring_full[stage],
                        h * 64, row_blk * kBlk, bh);
        pend_valid |= 1u << stage;
        pend_phase = (pend_phase & ~(1u << stage)) | (phase << stage);
        if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
        }
        return true;
    }
    __device__ __forceinline__ void drain(Bars* bars, int32_t fixed_pending) {
        volatile uint32_t never = 0;
        for (uint32_t s = 0; s < kStages; ++s)
            if (pend_valid & (1u << s))
                mbar_wait_bounded(&bars->ring_full[s], (pend_phase >> s) & 1u, &never, &g_fab_error_word, kErrDrain,
                                  1000000000ull);
        if (fixed_pending >= 0)
            mbar_wait_bounded(&bars->fixed_full, static_cast<uint32_t>(fixed_pending), &never, &g_fab_error_word,
                              kErrDrain, 1000000000ull);
    }
};

// The MMA warp's position in the ring (consumed in the producer's order by Issuer::ring_one).
struct RingWait {
    uint32_t stage = 0, phase = 0;
};

// Per-thread parities of the MMA warp's waits, kept across units.
struct MmaPar {
    uint32_t mid = 0, ds = 0;
};

// The MMA warp runs converged: every lane computes the same descriptors and waits on the same
// barriers (their give-up decisions ANDed over the warp), and only the elected lane issues the
// tcgen05.mma / tcgen05.commit instructions, predicated.  Warp-uniform descriptor values keep the
// issuing lane's stream between two MMAs short.
struct Issuer {
    uint32_t leader;
    __device__ __forceinline__ bool wait(uint64_t* bar, uint32_t parity, volatile uint32_t* abort_flag) const {
        const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, abort_flag, &g_fab_error_word, kErrMma));
        if (ok) tc_fence_after();
        return ok;
    }
    __device__ __forceinline__ bool wait_flip(uint64_t* bar, uint32_t& par, volatile uint32_t* abort_flag) const {
        if (!wait(bar, par, abort_flag)) return false;
        par ^= 1;
        return true;
    }
    __device__ __forceinline__ void commit(uint64_t* bar) const { tc_commit_if(leader, bar); }
    __device__ __forceinline__ void mma_ss(uint32_t d, Sw128Desc a, Sw128Desc b, uint32_t idesc, uint32_t acc) const {
        mma_ss2_if(leader, d, a, b, idesc, acc);
    }
    __device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a_tmem, Sw128Desc b, uint32_t idesc, uint32_t acc) const {
        mma_ts2_if(leader, d, a_tmem, b, idesc, acc);
    }
    // D (M=128, N=128) = A (128 x HD, K-major smem) * B^T (128 x HD, K-major smem): HD/16 K-steps.
    template <uint32_t HD>
    __device__ __forceinline__ void ss(uint32_t d_tmem, uint32_t a_addr, uint32_t b_addr, uint32_t idesc) const {
        const Sw128Desc ad = make_sw128_desc2(a_addr, 16, 1024), bd = make_sw128_desc2(b_addr, 16, 1024);
#pragma unroll
        for (uint32_t kk = 0; kk < HD / 16; ++kk) {
            const uint32_t off = ((kk >> 2) * kPanelBytes + (kk & 3) * 32) >> 4;
            mma_ss(d_tmem, Sw128Desc{ad.lo + off, ad.hi}, Sw128Desc{bd.lo + off, bd.hi}, idesc, kk > 0);
        }
    }
    // D (M=128, N=HD) (+)= A * B with B a 128-row MN-major smem tile (K along its rows) and A a
    // 128 x 128 16-bit tile in TMEM packed by the warpgroups: K range [kCols*g, kCols*(g+1)) in
    // columns [kCols*g, kCols*g + kCols/2) from `a_tmem`.  `accumulate` false starts D afresh.
    __device__ __forceinline__ void ts(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_addr, uint32_t idesc,
                                       bool accumulate) const {
        const Sw128Desc bd = make_sw128_desc2(b_addr, kPanelBytes, 1024);
#pragma unroll
        for (uint32_t kk = 0; kk < 8; ++kk)
            mma_ts(d_tmem, a_tmem + (kk / kStepsWG) * kCols + (kk % kStepsWG) * 8, Sw128Desc{bd.lo + kk * (2048 >> 4), bd.hi}, idesc,
                   (accumulate || kk > 0) ? 1u : 0u);
    }
    __device__ __forceinline__ bool ring_one(RingWait& ring, Bars* bars, volatile uint32_t* abort_flag,
                                             uint32_t& st) const {
        if (!wait(&bars->ring_full[ring.stage], ring.phase, abort_flag)) return false;
        st = ring.stage;
        if (++ring.stage == kStages) {
            ring.stage = 0;
            ring.phase ^= 1;
        }
        return true;
    }
    __device__ __forceinline__ void finish(Bars* bars) const {
        commit(&bars->mma_done);
        volatile uint32_t never = 0;
        mbar_wait_bounded(&bars->mma_done, 0, &never, &g_fab_error_word, kErrDrain, 1000000000ull);
    }
};

// Elementwise side: waits on an MMA barrier, decided for the whole warpgroup.
__device__ __forceinline__ bool ew_wait(uint32_t g, uint64_t* bar, uint32_t& par, volatile uint32_t* abort_flag) {
    if (!wg_all(g, mbar_wait_bounded(bar, par, abort_flag, &g_fab_error_word, kErrElem))) return false;
    par ^= 1;
    tc_fence_after();
    return true;
}

__device__ __forceinline__ void ew_arrive(uint64_t* bar) {
    tc_fence_before();
    mbar_arrive(bar);
}

// ============================================================================================
// dQ (and Delta)
// ============================================================================================
template <bool kBF16, uint32_t HD>
__global__ void __launch_bounds__(kThreads, 1)
    fa_bwd_dq_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                     const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                     const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    using D = Dims<HD>;
    Bars* bars = reinterpret_cast<Bars*>(smem + D::kOffBar);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + D::kOffBar + sizeof(Bars));
    volatile uint32_t* abort_flag = tmem_slot + 1;
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const uint32_t tmem_base = setup_cta(bars, tmem_slot, abort_flag, warp);
    const uint32_t sQ = smem_u32(smem + kOffFixed), sDO = sQ + D::kTileBytes, sRing = smem_u32(smem + D::kOffRing);
    const uint32_t tS = tmem_base, tDQ = tmem_base + 384;
    auto tDP = [&](uint32_t b) { return tmem_base + 128 + 128 * b; };
    if (warp == kTmaWarp) {
        if (lane == 0) {
            Ring ring;
            uint32_t it = 0;
            int32_t fixed_pending = -1;
            bool ok = true;
            Units u(blockIdx.x);
            uint32_t bh, qb;
            for (; ok && u.next(p, bh, qb); ++it) {
                if (!mbar_wait_bounded(&bars->fixed_empty, (it & 1) ^ 1, abort_flag, &g_fab_error_word, kErrProducer)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&bars->fixed_full, 2 * D::kTileBytes);
                for (uint32_t h = 0; h < D::kPanels; ++h) {
                    tma_load_3d(smem + kOffFixed + h * kPanelBytes, &tm_q, &bars->fixed_full, h * 64, qb * kBlk, bh);
                    tma_load_3d(smem + kOffFixed + D::kTileBytes + h * kPanelBytes, &tm_do, &bars->fixed_full, h * 64,
                                qb * kBlk, bh);
                }
                fixed_pending = static_cast<int32_t>(it & 1);
                const uint32_t nkv = kv_blocks_for(p, qb);
                // the MMA warp's order: K_0, V_0, then V_m ahead of K_m (dP runs a block ahead of S)
                ok = ring.template load<HD>(bars, smem, &tm_k, 0, bh, abort_flag) && ring.template load<HD>(bars, smem, &tm_v, 0, bh, abort_flag);
                for (uint32_t m = 1; m < nkv && ok; ++m)
                    ok = ring.template load<HD>(bars, smem, &tm_v, m, bh, abort_flag) && ring.template load<HD>(bars, smem, &tm_k, m, bh, abort_flag);
            }
            if (!ok) ring.drain(bars, fixed_pending);
        }
    } else if (warp == kMmaWarp) {
        {
            const Issuer is{elect_one() ? 1u : 0u};
            const uint32_t idesc_ss = make_idesc_f16(kBF16, 128, 128, false, false);
            const uint32_t idesc_ts = make_idesc_f16(kBF16, 128, HD, false, true);
            RingWait ring;
            MmaPar par;
            uint32_t it = 0;
            Units u(blockIdx.x);
            uint32_t bh, qb;
            for (; u.next(p, bh, qb); ++it) {
                const uint32_t n = kv_blocks_for(p, qb);
                if (!is.wait(&bars->fixed_full, it & 1, abort_flag)) break;
                tc_fence_after();
                uint32_t ks, vs;
                if (!is.ring_one(ring, bars, abort_flag, ks)) break;
                is.template ss<HD>(tS, sQ, sRing + ks * D::kTileBytes, idesc_ss);             // S_0 = Q K_0^T
                is.commit(&bars->s_full);
                bool ok = true;
                for (uint32_t b = 0; b < 2 && b < n && ok; ++b) {                // dP_0, dP_1 = dO V_b^T
                    if (!is.ring_one(ring, bars, abort_flag, vs)) { ok = false; break; }
                    is.template ss<HD>(tDP(b), sDO, sRing + vs * D::kTileBytes, idesc_ss);
                    is.commit(&bars->dp_full[b]);
                    is.commit(&bars->ring_empty[vs]);                            // V has no other reader
                }
                if (!ok) break;
                if (!is.wait(&bars->acc_empty, (it & 1) ^ 1, abort_flag)) break;
                for (uint32_t j = 0; j < n && ok; ++j) {
                    const bool nxt = j + 1 < n;
                    uint32_t kn = 0, vn = 0;
                    // S_j has been read into registers: the next S goes into its columns
                    if (!is.wait_flip(&bars->mid, par.mid, abort_flag)) { ok = false; break; }
                    if (nxt) {
                        if (!is.ring_one(ring, bars, abort_flag, kn)) { ok = false; break; }
                        is.template ss<HD>(tS, sQ, sRing + kn * D::kTileBytes, idesc_ss);
                        is.commit(&bars->s_full);
                    }
                    // dS_j packed over dP_j: dQ += dS_j K_j, then dP_{j+2} into that buffer
                    if (!is.wait_flip(&bars->ds_full, par.ds, abort_flag)) { ok = false; break; }
                    is.ts(tDQ, tDP(j & 1), sRing + ks * D::kTileBytes, idesc_ts, j > 0);
                    is.commit(&bars->ring_empty[ks]);
                    if (j + 2 < n) {
                        if (!is.ring_one(ring, bars, abort_flag, vn)) { ok = false; break; }
                        is.template ss<HD>(tDP(j & 1), sDO, sRing + vn * D::kTileBytes, idesc_ss);
                        is.commit(&bars->dp_full[j & 1]);
                        is.commit(&bars->ring_empty[vn]);
                    }
                    ks = kn;
                }
                if (!ok) break;
                is.commit(&bars->fixed_empty);
                is.commit(&bars->acc_full);
            }
            is.finish(bars);
        }
    } else {
        // ====== elementwise: Delta, P, dS, dQ epilogue (row = TMEM lane; warpgroup g = keys [kCols*g, kCols*(g+1))) ======
        const uint32_t t = threadIdx.x & 127, g = warp >> 2;
        const uint32_t lane_field = ((warp & 3) * 32) << 16;
        const uint8_t* tDOs = smem + kOffFixed + D::kTileBytes;
        uint32_t it = 0, s_par = 0, dp_par[2] = {0, 0}, acc_par = 0;
        bool ok = true;
        Units u(blockIdx.x);
        uint32_t bh, qb;
        while (ok && u.next(p, bh, qb)) {
            const uint32_t row = qb * kBlk + t;
            const bool valid = row < p.S_q;
            const size_t ridx = static_cast<size_t>(bh) * p.S_q + row;
            ok = wg_all(g, mbar_wait_bounded(&bars->fixed_full, it & 1, abort_flag, &g_fab_error_word, kErrElem));
            if (!ok) break;
            ++it;
            // Delta = rowsum(dO * O) of this row (dO from the staged tile, O from global); each
            // warpgroup forms it (the two run independently); warpgroup 0 stores it.
            float delta = 0.f, nlse2 = -INFINITY;
            if (valid) {
                const uint4* orow = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.o) + ridx * HD);
                float d2 = 0.f;
#pragma unroll 4
                for (uint32_t c = 0; c < HD / 8; ++c) {
                    const uint4 a = tile_chunk(tDOs, t, c), b = __ldg(orow + c);
                    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 x = unpack2<kBF16>(aw[e]), y = unpack2<kBF16>(bw[e]);
                        delta = fmaf(x.x, y.x, delta);
                        d2 = fmaf(x.y, y.y, d2);
                    }
                }
                delta += d2;
                nlse2 = -p.lse[ridx] * 1.4426950408889634f;
                if (g == 0) p.delta[ridx] = delta;
            }
            const uint32_t nkv = kv_blocks_for(p, qb);
            // on the diagonal block, key c of this warpgroup's columns is visible when kCols*g + c <= t
            const int32_t lim = static_cast<int32_t>(t) + 1 - static_cast<int32_t>(kCols * g);
            for (uint32_t j = 0; j < nkv; ++j) {
                // phase 1: S -> registers (then the MMA warp may overwrite it), P
                if (!(ok = ew_wait(g, &bars->s_full, s_par, abort_flag))) break;
                float pr[kCols];
                {
                    uint32_t s[kCols];
#pragma unroll
                    for (uint32_t c = 0; c < kChunks; ++c)
                        tmem_ld32(tS + kCols * g + 32 * c + lane_field, *reinterpret_cast<uint32_t(*)[32]>(s + 32 * c));
                    tmem_wait_ld();
                    ew_arrive(&bars->mid);
                    if (p.causal && j == qb) {
#pragma unroll
                        for (int c = 0; c < static_cast<int>(kCols); ++c)
                            pr[c] = c < lim ? ex2(fmaf(__uint_as_float(s[c]), p.scale_log2, nlse2)) : 0.f;
                    } else {
#pragma unroll
                        for (int c = 0; c < static_cast<int>(kCols); ++c)
                            pr[c] = ex2(fmaf(__uint_as_float(s[c]), p.scale_log2, nlse2));
                    }
                }
                // phase 2: dS = P (dP - Delta), packed over dP
                const uint32_t buf = j & 1;
                if (!(ok = ew_wait(g, &bars->dp_full[buf], dp_par[buf], abort_flag))) break;
#pragma unroll
                for (uint32_t c = 0; c < kChunks; ++c) {
                    uint32_t dp[32], pk[16];
                    tmem_ld32(tDP(buf) + kCols * g + 32 * c + lane_field, dp);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 16; ++e)
                        pk[e] = pack2<kBF16>(pr[32 * c + 2 * e] * (__uint_as_float(dp[2 * e]) - delta),
                                             pr[32 * c + 2 * e + 1] * (__uint_as_float(dp[2 * e + 1]) - delta));
                    tmem_st16(tDP(buf) + kCols * g + 16 * c + lane_field, pk);
                }
                tmem_wait_st();
                ew_arrive(&bars->ds_full);
            }
            if (!ok) break;
            if (!(ok = ew_wait(g, &bars->acc_full, acc_par, abort_flag))) break;
            // epilogue: dQ columns [kOutCols*g, kOutCols*(g+1)), scaled
            uint8_t* dq_row = static_cast<uint8_t*>(p.out0) + ridx * HD * 2;
            uint32_t acc[D::kOutChunks][32];
#pragma unroll
            for (uint32_t c = 0; c < D::kOutChunks; ++c) tmem_ld32(tDQ + D::kOutCols * g + 32 * c + lane_field, acc[c]);
            tmem_wait_ld();
            ew_arrive(&bars->acc_empty);
            if (valid) {
#pragma unroll
                for (uint32_t c = 0; c < D::kOutChunks; ++c) {
                    uint32_t pk[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e)
                        pk[e] = pack2<kBF16>(__uint_as_float(acc[c][2 * e]) * p.scale,
                                             __uint_as_float(acc[c][2 * e + 1]) * p.scale);
                    uint4* dst = reinterpret_cast<uint4*>(dq_row + (D::kOutCols * g + 32 * c) * 2);
#pragma unroll
                    for (int v = 0; v < 4; ++v) dst[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
                }
            }
        }
    }
    teardown_cta(tmem_base, warp);
}

// ============================================================================================
// dK, dV
// ============================================================================================
template <bool kBF16, uint32_t HD>
__global__ void __launch_bounds__(kThreads, 1)
    fa_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                       const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                       const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    using D = Dims<HD>;
    Bars* bars = reinterpret_cast<Bars*>(smem + D::kOffBar);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + D::kOffBar + sizeof(Bars));
    volatile uint32_t* abort_flag = tmem_slot + 1;
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const uint32_t nq = n_blocks(p.S_q);
    const uint32_t tmem_base = setup_cta(bars, tmem_slot, abort_flag, warp);
    const uint32_t sK = smem_u32(smem + kOffFixed), sV = sK + D::kTileBytes, sRing = smem_u32(smem + D::kOffRing);
    const uint32_t tS = tmem_base, tDP = tmem_base + 128, tDV = tmem_base + 256, tDK = tmem_base + 384;
    if (warp == kTmaWarp) {
        if (lane == 0) {
            Ring ring;
            uint32_t it = 0;
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
                mbar_arrive_expect_tx(&bars->fixed_full, 2 * D::kTileBytes);
                for (uint32_t h = 0; h < D::kPanels; ++h) {
                    tma_load_3d(smem + kOffFixed + h * kPanelBytes, &tm_k, &bars->fixed_full, h * 64, kb * kBlk, bh);
                    tma_load_3d(smem + kOffFixed + D::kTileBytes + h * kPanelBytes, &tm_v, &bars->fixed_full, h * 64,
                                kb * kBlk, bh);
                }
                fixed_pending = static_cast<int32_t>(it & 1);
                ++it;
                for (uint32_t i = q0; i < nq && ok; ++i)  // Q_i, then dO_i
                    ok = ring.template load<HD>(bars, smem, &tm_q, i, bh, abort_flag) && ring.template load<HD>(bars, smem, &tm_do, i, bh, abort_flag);
            }
            if (!ok) ring.drain(bars, fixed_pending);
        }
    } else if (warp == kMmaWarp) {
        {
            const Issuer is{elect_one() ? 1u : 0u};
            const uint32_t idesc_ss = make_idesc_f16(kBF16, 128, 128, false, false);
            const uint32_t idesc_ts = make_idesc_f16(kBF16, 128, HD, false, true);
            RingWait ring;
            MmaPar par;
            uint32_t it = 0;
            Units u(blockIdx.x);
            uint32_t bh, kb;
            while (u.next(p, bh, kb)) {
                const uint32_t q0 = q_first_for(p, kb);
                if (q0 >= nq) continue;  // the producer skipped this unit too
                if (!is.wait(&bars->fixed_full, it & 1, abort_flag)) break;
                tc_fence_after();
                uint32_t qs, os;
                if (!is.ring_one(ring, bars, abort_flag, qs)) break;
                is.template ss<HD>(tS, sK, sRing + qs * D::kTileBytes, idesc_ss);             // S^T = K Q_q0^T
                is.commit(&bars->s_full);
                if (!is.ring_one(ring, bars, abort_flag, os)) break;
                is.template ss<HD>(tDP, sV, sRing + os * D::kTileBytes, idesc_ss);            // dP^T = V dO_q0^T
                is.commit(&bars->dp_full[0]);
                if (!is.wait(&bars->acc_empty, (it & 1) ^ 1, abort_flag)) break;
                bool ok = true;
                for (uint32_t i = q0; i < nq && ok; ++i) {
                    const bool nxt = i + 1 < nq;
                    uint32_t qn = 0, on = 0;
                    // P^T_i packed over S^T: dV += P^T dO_i, then the next S^T
                    if (!is.wait_flip(&bars->mid, par.mid, abort_flag)) { ok = false; break; }
                    is.ts(tDV, tS, sRing + os * D::kTileBytes, idesc_ts, i > q0);
                    is.commit(&bars->ring_empty[os]);                            // dO_i is done
                    if (nxt) {
                        if (!is.ring_one(ring, bars, abort_flag, qn)) { ok = false; break; }
                        is.template ss<HD>(tS, sK, sRing + qn * D::kTileBytes, idesc_ss);
                        is.commit(&bars->s_full);
                    }
                    // dS^T_i packed over dP^T: dK += dS^T Q_i, then the next dP^T
                    if (!is.wait_flip(&bars->ds_full, par.ds, abort_flag)) { ok = false; break; }
                    is.ts(tDK, tDP, sRing + qs * D::kTileBytes, idesc_ts, i > q0);
                    is.commit(&bars->ring_empty[qs]);                            // Q_i is done
                    if (nxt) {
                        if (!is.ring_one(ring, bars, abort_flag, on)) { ok = false; break; }
                        is.template ss<HD>(tDP, sV, sRing + on * D::kTileBytes, idesc_ss);
                        is.commit(&bars->dp_full[0]);
                    }
                    qs = qn;
                    os = on;
                }
                if (!ok) break;
                is.commit(&bars->fixed_empty);
                is.commit(&bars->acc_full);
                ++it;
            }
            is.finish(bars);
        }
    } else {
        // ====== elementwise: P^T, dS^T, dK/dV epilogue (key = TMEM lane; warpgroup g = queries [kCols*g, kCols*(g+1))) ======
        const uint32_t t = threadIdx.x & 127, g = warp >> 2;
        const uint32_t lane_field = ((warp & 3) * 32) << 16;
        // this warpgroup's staging: [0, kCols) -lse*log2(e), [kCols, 2 kCols) Delta of its queries
        float* vec = reinterpret_cast<float*>(smem + D::kOffVec) + g * 2 * kCols;
        uint32_t s_par = 0, dp_par = 0, acc_par = 0;
        Units u(blockIdx.x);
        uint32_t bh, kb;
        bool ok = true;
        // on the diagonal block, query c of this warpgroup's columns sees the key when kCols*g + c >= t
        const int32_t first = static_cast<int32_t>(t) - static_cast<int32_t>(kCols * g);
        while (ok && u.next(p, bh, kb)) {
            const uint32_t key = kb * kBlk + t;
            const size_t kidx = static_cast<size_t>(bh) * p.S_k + key;
            const uint32_t q0 = q_first_for(p, kb);
            if (q0 < nq) {
                for (uint32_t i = q0; i < nq; ++i) {
                    // stage -lse*log2(e) (-inf past S_q, so P = 0 there) and Delta of this warpgroup's
                    // queries, once every thread of the group is done with the previous block's
                    const uint32_t r = i * kBlk + kCols * g + (t % kCols);
                    const size_t ridx = static_cast<size_t>(bh) * p.S_q + r;
                    wg_sync(g);
                    if (t < kCols)
                        vec[t] = r < p.S_q ? -p.lse[ridx] * 1.4426950408889634f : -INFINITY;
                    else if (t < 2 * kCols)
                        vec[t] = r < p.S_q ? p.delta[ridx] : 0.f;
                    // phase 1: P^T from S^T, packed over it (the wait also publishes the staged values)
                    if (!(ok = ew_wait(g, &bars->s_full, s_par, abort_flag))) break;
                    float pr[kCols];
                    {
                        uint32_t s[kCols], pk[kCols / 2];
#pragma unroll
                        for (uint32_t c = 0; c < kChunks; ++c)
                            tmem_ld32(tS + kCols * g + 32 * c + lane_field, *reinterpret_cast<uint32_t(*)[32]>(s + 32 * c));
                        const float4* nl4 = reinterpret_cast<const float4*>(vec);
                        tmem_wait_ld();
                        if (p.causal && i == kb) {
#pragma unroll
                            for (int e4 = 0; e4 < static_cast<int>(kCols / 4); ++e4) {
                                const float4 nl = nl4[e4];
                                const float nla[4] = {nl.x, nl.y, nl.z, nl.w};
#pragma unroll
                                for (int k = 0; k < 4; ++k) {
                                    const int c = 4 * e4 + k;
                                    pr[c] = c >= first ? ex2(fmaf(__uint_as_float(s[c]), p.scale_log2, nla[k])) : 0.f;
                                }
                            }
                        } else {
#pragma unroll
                            for (int e4 = 0; e4 < static_cast<int>(kCols / 4); ++e4) {
                                const float4 nl = nl4[e4];
                                const float nla[4] = {nl.x, nl.y, nl.z, nl.w};
#pragma unroll
                                for (int k = 0; k < 4; ++k)
                                    pr[4 * e4 + k] = ex2(fmaf(__uint_as_float(s[4 * e4 + k]), p.scale_log2, nla[k]));
                            }
                        }
#pragma unroll
                        for (int e = 0; e < static_cast<int>(kCols / 2); ++e) pk[e] = pack2<kBF16>(pr[2 * e], pr[2 * e + 1]);
#pragma unroll
                        for (uint32_t c = 0; c < kChunks; ++c) tmem_st16(tS + kCols * g + 16 * c + lane_field, pk + 16 * c);
                        tmem_wait_st();
                        ew_arrive(&bars->mid);
                    }
                    // phase 2: dS^T = P^T (dP^T - Delta), packed over dP^T
                    if (!(ok = ew_wait(g, &bars->dp_full[0], dp_par, abort_flag))) break;
#pragma unroll
                    for (uint32_t c = 0; c < kChunks; ++c) {
                        uint32_t dp[32], pk[16];
                        tmem_ld32(tDP + kCols * g + 32 * c + lane_field, dp);
                        const float4* dl4 = reinterpret_cast<const float4*>(vec + kCols + 32 * c);
                        tmem_wait_ld();
#pragma unroll
                        for (int e4 = 0; e4 < 8; ++e4) {
                            const float4 dl = dl4[e4];
                            const int b = 32 * c + 4 * e4;
                            pk[2 * e4] = pack2<kBF16>(pr[b] * (__uint_as_float(dp[4 * e4]) - dl.x),
                                                      pr[b + 1] * (__uint_as_float(dp[4 * e4 + 1]) - dl.y));
                            pk[2 * e4 + 1] = pack2<kBF16>(pr[b + 2] * (__uint_as_float(dp[4 * e4 + 2]) - dl.z),
                                                          pr[b + 3] * (__uint_as_float(dp[4 * e4 + 3]) - dl.w));
                        }
                        tmem_st16(tDP + kCols * g + 16 * c + lane_field, pk);
                    }
                    tmem_wait_st();
                    ew_arrive(&bars->ds_full);
                }
                if (!ok) break;
                if (!(ok = ew_wait(g, &bars->acc_full, acc_par, abort_flag))) break;
            }
            // epilogue: dV, dK (scaled) of this key, columns [kOutCols*g, kOutCols*(g+1)); zeros when no query sees the block
            const bool valid = key < p.S_k;
            uint8_t* dk_row = static_cast<uint8_t*>(p.out0) + kidx * HD * 2;
            uint8_t* dv_row = static_cast<uint8_t*>(p.out1) + kidx * HD * 2;
#pragma unroll 1
            for (uint32_t c = 0; c < D::kOutChunks; ++c) {
                uint32_t av[32], ak[32], pv[16], pk[16];
                if (q0 < nq) {
                    tmem_ld32(tDV + D::kOutCols * g + 32 * c + lane_field, av);
                    tmem_ld32(tDK + D::kOutCols * g + 32 * c + lane_field, ak);
                    tmem_wait_ld();
                    if (c + 1 == D::kOutChunks) ew_arrive(&bars->acc_empty);  // the accumulators are read: the next unit may start them
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
                    uint4* dv = reinterpret_cast<uint4*>(dv_row + (D::kOutCols * g + 32 * c) * 2);
                    uint4* dk = reinterpret_cast<uint4*>(dk_row + (D::kOutCols * g + 32 * c) * 2);
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        dv[v] = make_uint4(pv[4 * v], pv[4 * v + 1], pv[4 * v + 2], pv[4 * v + 3]);
                        dk[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
                    }
                }
            }
        }
    }
    teardown_cta(tmem_base, warp);
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

template <bool kBF16, uint32_t HD>
int launch_tc(const void* q, const void* k, const void* v, const void* o, const void* dO, const float* lse, void* dq,
              void* dk, void* dv, float* delta, const flash_attention_fwd_fused_tiling_data* t, cudaStream_t stream) {
    static std::once_flag reg_once;
    std::call_once(reg_once, [] { register_error_word(read_error_word); });
    const uint64_t BH = static_cast<uint64_t>(t->B) * t->H;
    const CUtensorMapDataType dt = kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const uint32_t box[3] = {64, 128, 1};
    CUtensorMap tmq, tmdo, tmk, tmv;
    using D = Dims<HD>;
    {
        uint64_t dims[3] = {HD, t->S_q, BH};
        uint64_t strides[2] = {HD * 2, static_cast<uint64_t>(t->S_q) * HD * 2};
        if (int rc = encode_tmap(&tmq, dt, 3, q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
        if (int rc = encode_tmap(&tmdo, dt, 3, dO, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
    }
    {
        uint64_t dims[3] = {HD, t->S_k, BH};
        uint64_t strides[2] = {HD * 2, static_cast<uint64_t>(t->S_k) * HD * 2};
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
        const void* fn = pass == 0 ? reinterpret_cast<const void*>(fa_bwd_dq_kernel<kBF16, HD>)
                                   : reinterpret_cast<const void*>(fa_bwd_dkdv_kernel<kBF16, HD>);
        if (int rc = set_max_dynamic_smem(fn, D::kSmemBytes, pass == 0 ? "fa_bwd_dq_kernel" : "fa_bwd_dkdv_kernel"))
            return rc;
        prm.n_blk = pass == 0 ? (t->S_q + kBlk - 1) / kBlk : (t->S_k + kBlk - 1) / kBlk;
        prm.num_pairs = static_cast<uint32_t>(BH * ((prm.n_blk + 1) / 2));
        prm.out0 = pass == 0 ? dq : dk;
        prm.out1 = dv;
        uint32_t grid = static_cast<uint32_t>(sm_count());
        if (grid > prm.num_pairs) grid = prm.num_pairs;
        if (pass == 0)
            fa_bwd_dq_kernel<kBF16, HD><<<grid, kThreads, D::kSmemBytes, stream>>>(tmq, tmdo, tmk, tmv, prm);
        else
            fa_bwd_dkdv_kernel<kBF16, HD><<<grid, kThreads, D::kSmemBytes, stream>>>(tmq, tmdo, tmk, tmv, prm);
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
    const bool tc_shape = t->D == t->D_v && (t->D == 128 || t->D == 64) && t->scale > 0.f && aligned16(q) &&
                          aligned16(k) && aligned16(v) && aligned16(o) && aligned16(dO) && aligned16(dq) &&
                          aligned16(dk) && aligned16(dv);
    if (dtype == HC_DTYPE_BF16) {
        if (!tc_shape) return fab::launch_simt<bf16_t>(q, k, v, o, dO, lse, dq, dk, dv, delta, t, s);
        return t->D == 128 ? fab::launch_tc<true, 128>(q, k, v, o, dO, lse, dq, dk, dv, delta, t, s)
                           : fab::launch_tc<true, 64>(q, k, v, o, dO, lse, dq, dk, dv, delta, t, s);
    }
    if (dtype == HC_DTYPE_F16) {
        if (!tc_shape) return fab::launch_simt<f16_t>(q, k, v, o, dO, lse, dq, dk, dv, delta, t, s);
        return t->D == 128 ? fab::launch_tc<false, 128>(q, k, v, o, dO, lse, dq, dk, dv, delta, t, s)
                           : fab::launch_tc<false, 64>(q, k, v, o, dO, lse, dq, dk, dv, delta, t, s);
    }
    return fab::launch_simt<float>(q, k, v, o, dO, lse, dq, dk, dv, delta, t, s);
}

extern "C" int hc_flash_attention_bwd_last_path(void) { return fab::t_last_path; }
