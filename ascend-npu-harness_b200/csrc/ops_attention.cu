// flash_attention_fwd_fused on B200.
//
// Algorithm: the reference golden's online softmax
// (ops/flash_attention_fwd_fused/golden/flash_attention_fwd_fused_golden.cpp:26-107):
// per query row keep a running max m and sum l, rescale the accumulator when m grows,
// O = acc / l; causal masking hides key k from query q when k > q (golden.cpp:61-66).
// Added output: lse = m + ln(l) per row (natural log), the standard flash-attention residual.
//
// Tensor-core path (bf16/fp16, D = HD and D_v = HDV, each 128 or 64), one persistent CTA per SM:
//   * a CTA work unit is (b*h, block of 256 query rows) = two 128-row Q tiles;
//   * warp 9 (producer) streams Q tiles and 128-key K/V tiles into shared memory with TMA
//     (128-byte swizzle, a 4-stage K/V ring at HD 128 and 8 stages at HD 64, no multicast);
//   * warp 8 (one thread) issues tcgen05.mma: S_i = Q_i K^T into TMEM (M=128, N=128, K=16 x HD/16)
//     and O_i += P_i V (N = HDV) with P read straight from TMEM (the "TS" form), V as an MN-major
//     operand;
//   * warpgroups 0 and 1 each own one Q tile: thread t owns row t (TMEM lane t), reads its S row
//     with tcgen05.ld, applies the causal / sequence-tail mask, updates (m, l) in the log2
//     domain, writes P (16-bit) back over its S row with tcgen05.st, and rescales its O row in
//     TMEM only when the running max grew by more than 2^8 (lazy rescaling: exact, because O and
//     l always refer to the same m);
//   * the two Q tiles ping-pong: the tensor core runs one tile's MMAs while the other tile's
//     softmax runs on the CUDA cores;
//   * the epilogue (O / l -> 16-bit, lse) is done by the owning warpgroup from TMEM.
// TMEM: S0 [0,128) S1 [128,256) O0 [256,256+HDV) O1 [384,384+HDV) columns; P_i overlays S_i.
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
#include <type_traits>

#include "hc_device.cuh"
#include "hc_internal.h"
#include "exp2_poly.cuh"
#include "sm100.cuh"
#include "tmap.h"

namespace hc {
namespace fa {

using namespace sm100;

constexpr uint32_t kBM = 128;      // query rows per Q tile
constexpr uint32_t kBN = 128;      // keys per K/V tile
constexpr uint32_t kThreads = 384;
constexpr uint32_t kPanelBytes = kBM * 64 * 2;  // one 64-column swizzle panel of a 128-row tile: 16 KB
constexpr float kRescaleThreshold = 8.0f;       // log2 units

// Shared-memory geometry for Q/K head dimension HD and V/O head dimension HDV (each 64 or 128).
// A tile is 128 rows of 16-bit elements stored as 64-column panels of 128-byte swizzled rows;
// K and V tiles alternate in one ring whose slots hold the larger of the two, and the ring is
// deeper when slots are smaller.
template <uint32_t HD, uint32_t HDV>
struct Geom {
    static_assert((HD == 64 || HD == 128) && (HDV == 64 || HDV == 128), "head dims 64 and 128");
    static constexpr uint32_t kPanels = HD / 64;    // Q and K tiles
    static constexpr uint32_t kPanelsV = HDV / 64;  // V tiles
    static constexpr uint32_t kTileBytes = kPanels * kPanelBytes;
    static constexpr uint32_t kTileBytesV = kPanelsV * kPanelBytes;
    static constexpr uint32_t kSlotBytes = kTileBytes > kTileBytesV ? kTileBytes : kTileBytesV;
    static constexpr uint32_t kStages = kSlotBytes == kPanelBytes ? 8 : 4;  // K/V ring depth
    static constexpr uint32_t kOffQ = 0;
    static constexpr uint32_t kOffKV = 2 * kTileBytes;
    static constexpr uint32_t kOffBar = kOffKV + kStages * kSlotBytes;
    static constexpr uint32_t kSmemBytes = kOffBar + 256 + 1024;  // + barriers/misc + alignment slack
};

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
    uint32_t S_q, S_k, BH, n_qblk, num_pairs;  // num_pairs = BH * ceil(n_qblk / 2)
    uint32_t group;    // query heads per K/V head: K/V head of flattened query head bh is bh / group
    float scale_log2;  // softmax scale * log2(e), > 0
    uint32_t causal;
};

template <uint32_t kStages>
struct Bars {
    uint64_t q_full, q_empty;
    uint64_t kv_full[kStages], kv_empty[kStages];
    uint64_t s_full[2], p_full[2], o_full[2];
    uint64_t mma_done;
};

// The work units (head, 256-row query block) of this CTA.  Units are handed out as pairs
// (qb, n_qblk-1-qb) of the same head: under the causal mask the two blocks of a pair need
// n_qblk+1 key tiles together whatever qb is, so a static round-robin over pairs gives every CTA
// the same work (to within one pair) without a scheduler in global memory.  Pairs are numbered
// head-major, so the CTAs in flight work on a few consecutive heads whose K/V tiles are fetched
// from HBM once and then served from L2.  The longer block of a pair comes first.
struct UnitSeq {
    uint32_t pi = blockIdx.x;
    uint32_t second = 0;
    __device__ __forceinline__ bool next(const Params& p, uint32_t& bh, uint32_t& qb) {
        const uint32_t per_head = (p.n_qblk + 1) / 2;
        while (pi < p.num_pairs) {
            bh = pi / per_head;
            const uint32_t j = pi - bh * per_head;
            if (!second) {
                second = 1;
                qb = p.n_qblk - 1 - j;
                return true;
            }
            second = 0;
            pi += gridDim.x;
            if (j != p.n_qblk - 1 - j) {  // the middle block of an odd count has no partner
                qb = j;
                return true;
            }
        }
        return false;
    }
};

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

__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// Register split: the CTA is launched with 168 registers/thread (384 threads x 168 = 64512, the
// per-SM file allows no more with 12 warps); the two softmax warpgroups then grow to
// HC_FA_REGS_SOFTMAX (each thread keeps a whole 128-key score row in registers) and the
// producer/MMA warpgroup shrinks to HC_FA_REGS_CTRL.  ptxas allocates each region with its own
// budget.
#ifndef HC_FA_REGS_SOFTMAX
#define HC_FA_REGS_SOFTMAX 208
#endif
#ifndef HC_FA_REGS_CTRL
#define HC_FA_REGS_CTRL 88
#endif
static_assert(2 * 128 * HC_FA_REGS_SOFTMAX + 128 * HC_FA_REGS_CTRL <= 384 * 168,
              "register split exceeds the registers the CTA is launched with");
static_assert(HC_FA_REGS_SOFTMAX % 8 == 0 && HC_FA_REGS_CTRL % 8 == 0, "setmaxnreg counts are multiples of 8");

template <int N>
__device__ __forceinline__ void reg_alloc() {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void reg_dealloc() {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// Pairs (c, c+1) of a 128-key row may be computed with the FMA-pipe exponential instead of MUFU
// ex2: bit (pair % 8) of the mask selects them.  At D = 64 each score carries half the MMA work of
// D = 128 while the softmax stream is the same, so the softmax bounds the kernel and moving 1/4 of
// the exponentials (pairs 0 and 4 of every 8) off MUFU measured +4-5 % on B200.  At D = 128 the
// tensor pipe's own efficiency bounds the step and every split measured slower, so none is used.
template <uint32_t HD>
__device__ __forceinline__ constexpr uint32_t poly_mask() { return HD == 64 ? 0x11u : 0x00u; }
// bit (pair % 8) of the mask set -> that pair uses the FMA-pipe exponential
template <uint32_t HD>
__device__ __forceinline__ constexpr bool poly_pair(int pair) { return (poly_mask<HD>() >> (pair & 7)) & 1; }

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

// Descriptor bases are built once per call; each K-step adds its byte offset >> 4 to the low
// word.  The MMAs are issued by one thread as a dependent chain, and a per-step rebuild of both
// 64-bit descriptors made that chain long enough to leave the tensor pipe idle after each
// softmax hand-off (4-5 % of the kernel's throughput on B200).
template <uint32_t HD>
__device__ __forceinline__ void issue_qk(uint32_t d_tmem, uint32_t q_addr, uint32_t k_addr, uint32_t idesc) {
    const Sw128Desc qd = make_sw128_desc2(q_addr, 16, 1024), kd = make_sw128_desc2(k_addr, 16, 1024);
#pragma unroll
    for (uint32_t kk = 0; kk < HD / 16; ++kk) {
        // K-step kk: 16 columns = 32 B inside a 128-B swizzle row; the second 64-column half
        // of the head lives kPanelBytes further on.
        const uint32_t off = ((kk >> 2) * kPanelBytes + (kk & 3) * 32) >> 4;
        mma_ss2(d_tmem, Sw128Desc{qd.lo + off, qd.hi}, Sw128Desc{kd.lo + off, kd.hi}, idesc, kk > 0);
    }
}

__device__ __forceinline__ void issue_pv(uint32_t o_tmem, uint32_t p_tmem, uint32_t v_addr, uint32_t idesc,
                                         bool accumulate) {
    const Sw128Desc vd = make_sw128_desc2(v_addr, kPanelBytes, 1024);
#pragma unroll
    for (uint32_t kk = 0; kk < kBN / 16; ++kk) {
        // 16 keys = 16 rows of the MN-major V panel = 2 swizzle atoms (2048 B); P: 8 columns.
        mma_ts2(o_tmem, p_tmem + kk * 8, Sw128Desc{vd.lo + kk * (2048 >> 4), vd.hi}, idesc,
                (accumulate || kk > 0) ? 1u : 0u);
    }
}

template <bool kBF16, uint32_t HD, uint32_t HDV>
__global__ void __launch_bounds__(kThreads, 1)
    fa_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const Params p) {
    using G = Geom<HD, HDV>;
    constexpr uint32_t kTileBytes = G::kTileBytes, kSlotBytes = G::kSlotBytes, kStages = G::kStages, kOffQ = G::kOffQ,
                       kOffKV = G::kOffKV, kOffBar = G::kOffBar;
    using BarsT = Bars<kStages>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    BarsT* bars = reinterpret_cast<BarsT*>(smem + kOffBar);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffBar + sizeof(BarsT));
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

    if (warp >= 8) {
        reg_dealloc<HC_FA_REGS_CTRL>();
    if (warp == 9) {
        // ===================================== producer =====================================
        if (lane == 0) {
            uint32_t stage = 0, phase = 0, q_iter = 0;
            // Copies issued but possibly still in flight: bit s of pend_valid / pend_phase holds
            // stage s's last load and the barrier phase it completes (bitmasks, not arrays, so
            // nothing is indexed dynamically in local memory).
            uint32_t pend_valid = 0, pend_phase = 0;
            int32_t q_pending = -1;
            bool ok = true;
            UnitSeq seq;
            uint32_t bh, qb;
            for (; ok && seq.next(p, bh, qb); ++q_iter) {
                const uint32_t row0 = qb * 2 * kBM;
                const uint32_t nkv = kv_tiles_for(p, row0 + kBM);
                if (!mbar_wait_bounded(&bars->q_empty, (q_iter & 1) ^ 1, abort_flag, &g_fa_error_word, kErrProducerQ)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&bars->q_full, 2 * kTileBytes);
                for (uint32_t i = 0; i < 2; ++i)
                    for (uint32_t h = 0; h < G::kPanels; ++h)
                        tma_load_3d(smem + kOffQ + i * kTileBytes + h * kPanelBytes, &tm_q, &bars->q_full,
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
                        mbar_arrive_expect_tx(&bars->kv_full[stage], kv ? G::kTileBytesV : kTileBytes);
                        for (uint32_t h = 0; h < (kv ? G::kPanelsV : G::kPanels); ++h)
                            tma_load_3d(smem + kOffKV + stage * kSlotBytes + h * kPanelBytes, kv ? &tm_v : &tm_k,
                                        &bars->kv_full[stage], static_cast<int32_t>(h * 64),
                                        static_cast<int32_t>(j * kBN), static_cast<int32_t>(bh / p.group));
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
                // Drain: every TMA copy issued must land before the CTA's shared memory is released.
                volatile uint32_t never = 0;
                for (uint32_t s = 0; s < kStages; ++s)
                    if (pend_valid & (1u << s))
                        mbar_wait_bounded(&bars->kv_full[s], (pend_phase >> s) & 1u, &never, &g_fa_error_word,
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
            const uint32_t idesc_pv = make_idesc_f16(kBF16, kBM, HDV, false, true);
            const uint32_t tS[2] = {tmem_base, tmem_base + 128};
            const uint32_t tO[2] = {tmem_base + 256, tmem_base + 384};
            const uint32_t qa[2] = {sQ, sQ + kTileBytes};
            uint32_t stage = 0, phase = 0, q_iter = 0;
            uint32_t p_par0 = 0, p_par1 = 0;
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
                uint32_t& par = i ? p_par1 : p_par0;
                if (!mbar_wait_bounded(&bars->p_full[i], par, abort_flag, &g_fa_error_word, kErrMmaP)) return false;
                par ^= 1;
                tc_fence_after();
                return true;
            };
            UnitSeq seq;
            uint32_t bh, qb;
            for (; ok && seq.next(p, bh, qb); ++q_iter) {
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
                issue_qk<HD>(tS[0], qa[0], sKV + kst * kSlotBytes, idesc_qk);
                tc_commit(&bars->s_full[0]);
                issue_qk<HD>(tS[1], qa[1], sKV + kst * kSlotBytes, idesc_qk);
                tc_commit(&bars->s_full[1]);
                tc_commit(&bars->kv_empty[kst]);
                if (nkv == 1) tc_commit(&bars->q_empty);
                for (uint32_t j = 1; j < nkv; ++j) {
                    if (!wait_kv(vst)) { ok = false; break; }            // V_{j-1}
                    if (j - 1 < n0) {
                        if (!wait_p(0)) { ok = false; break; }
                        issue_pv(tO[0], tS[0], sKV + vst * kSlotBytes, idesc_pv, j - 1 > 0);
                    }
                    if (!wait_kv(kst)) { ok = false; break; }            // K_j
                    if (j < n0) {
                        issue_qk<HD>(tS[0], qa[0], sKV + kst * kSlotBytes, idesc_qk);
                        tc_commit(&bars->s_full[0]);
                    }
                    if (!wait_p(1)) { ok = false; break; }
                    issue_pv(tO[1], tS[1], sKV + vst * kSlotBytes, idesc_pv, j - 1 > 0);
                    tc_commit(&bars->kv_empty[vst]);
                    issue_qk<HD>(tS[1], qa[1], sKV + kst * kSlotBytes, idesc_qk);
                    tc_commit(&bars->s_full[1]);
                    tc_commit(&bars->kv_empty[kst]);
                    if (j + 1 == nkv) tc_commit(&bars->q_empty);
                }
                if (!ok) break;
                if (!wait_kv(vst)) { ok = false; break; }                // V_{nkv-1}
                if (n0 == nkv) {
                    if (!wait_p(0)) { ok = false; break; }
                    issue_pv(tO[0], tS[0], sKV + vst * kSlotBytes, idesc_pv, nkv > 1);
                }
                tc_commit(&bars->o_full[0]);
                if (!wait_p(1)) { ok = false; break; }
                issue_pv(tO[1], tS[1], sKV + vst * kSlotBytes, idesc_pv, nkv > 1);
                tc_commit(&bars->o_full[1]);
                tc_commit(&bars->kv_empty[vst]);
            }
            // All issued MMAs must complete before TMEM is freed (normal and abort paths alike).
            tc_commit(&bars->mma_done);
            volatile uint32_t never = 0;
            mbar_wait_bounded(&bars->mma_done, 0, &never, &g_fa_error_word, kErrDrain, 1000000000ull);
        }
    }
    } else {
        reg_alloc<HC_FA_REGS_SOFTMAX>();
        // ============================== softmax / epilogue ===============================
        const uint32_t wg = warp / 4;                 // Q tile owned by this warpgroup
        const uint32_t r_local = threadIdx.x - wg * 128;  // row within the tile = TMEM lane
        const uint32_t lane_field = ((warp & 3) * 32) << 16;
        const uint32_t tS = tmem_base + wg * 128 + lane_field;
        const uint32_t tO = tmem_base + 256 + wg * 128 + lane_field;
        uint32_t s_par = 0, o_par = 0;
        UnitSeq seq;
        uint32_t bh, qb;
        while (seq.next(p, bh, qb)) {
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
                const uint32_t kbase = j * kBN;
                // Valid keys of this tile for this row: causal (k <= row) and sequence tail (k < S_k).
                int32_t lim = static_cast<int32_t>(p.S_k) - static_cast<int32_t>(kbase);
                if (p.causal) {
                    int32_t lc = static_cast<int32_t>(row) - static_cast<int32_t>(kbase) + 1;
                    if (lc < lim) lim = lc;
                }
                // Warp-uniform: masked tiles (the causal diagonal, the sequence tail) use MUFU
                // ex2 for every element so that masked keys give exactly 0.
                const bool masked = __any_sync(0xffffffffu, lim < static_cast<int32_t>(kBN));
                // The whole 128-key row of S comes out of TMEM in one round trip (four loads, one
                // wait) and stays in registers (the warpgroup's setmaxnreg budget allows it).
                uint32_t sr[128];
#pragma unroll
                for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, *reinterpret_cast<uint32_t(*)[32]>(sr + c * 32));
                tmem_wait_ld();
                if (masked) {
#pragma unroll
                    for (int c = 0; c < 128; ++c) sr[c] = (c < lim) ? sr[c] : __float_as_uint(-INFINITY);
                }
                // Row max: 3-input max in four independent chains.
                float mx4[4] = {__uint_as_float(sr[0]), __uint_as_float(sr[1]), __uint_as_float(sr[2]),
                                __uint_as_float(sr[3])};
#pragma unroll
                for (int pr = 2; pr < 64; ++pr)
                    mx4[pr & 3] = fmax3(mx4[pr & 3], __uint_as_float(sr[2 * pr]), __uint_as_float(sr[2 * pr + 1]));
                const float mx = fmaxf(fmax3(mx4[0], mx4[1], mx4[2]), mx4[3]);
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
                    for (int c = 0; c < static_cast<int>(HDV / 32); ++c) {
                        uint32_t orow[32];
                        tmem_ld32(tO + c * 32, orow);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 32; ++e) orow[e] = __float_as_uint(__uint_as_float(orow[e]) * alpha);
                        tmem_st32(tO + c * 32, orow);
                    }
                }
                const float neg_m = (m == -INFINITY) ? 0.f : -m;
                const float2 scale2 = make_float2(p.scale_log2, p.scale_log2);
                const float2 negm2 = make_float2(neg_m, neg_m);
                float2 lsum2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
                // Exponentials 32 keys at a time; each chunk's 16 packed P columns are written back
                // over S columns already read into registers.  kPoly: the FMA-pipe exponential for
                // the pairs poly_mask selects (unmasked tiles only: masked keys need an exact 0).
                // The masked / unmasked choice is made once per tile, outside the unrolled loop,
                // so that each variant is one straight-line block the scheduler can interleave.
                auto exp_tile = [&](auto poly_tag) {
                    constexpr bool kPoly = decltype(poly_tag)::value;
#pragma unroll
                    for (int g = 0; g < 4; ++g) {
                        uint32_t pk[16];
#pragma unroll
                        for (int q = 0; q < 16; ++q) {
                            const int pr = g * 16 + q;
                            // x = s * scale * log2(e) - m, two keys per packed FMA
                            float2 x = __ffma2_rn(
                                make_float2(__uint_as_float(sr[2 * pr]), __uint_as_float(sr[2 * pr + 1])), scale2, negm2);
                            if (kPoly && poly_pair<HD>(pr)) {
                                x = exp2_poly2(x);
                            } else {
                                x.x = ex2(x.x);
                                x.y = ex2(x.y);
                            }
                            lsum2[q & 1] = __fadd2_rn(lsum2[q & 1], x);
                            pk[q] = pack2<kBF16>(x.x, x.y);
                        }
                        tmem_st16(tS + g * 16, pk);
                    }
                };
                if constexpr (poly_mask<HD>() != 0) {
                    if (!masked)
                        exp_tile(std::true_type{});
                    else
                        exp_tile(std::false_type{});
                } else {
                    exp_tile(std::false_type{});
                }
                l += (lsum2[0].x + lsum2[0].y) + (lsum2[1].x + lsum2[1].y);
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
            uint8_t* orow_g = static_cast<uint8_t*>(p.o) + (static_cast<size_t>(bh) * p.S_q + row) * HDV * 2;
#pragma unroll
            for (int c = 0; c < static_cast<int>(HDV / 32); ++c) {
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
                                                          uint32_t causal, uint32_t group) {
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
                const T* krow = k + (bh / group * S_k + kj) * D;
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
                const T* vrow = v + (bh / group * S_k + k0 + jj) * Dv;
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

template <bool kBF16, uint32_t HD, uint32_t HDV>
int launch_tc(const void* q, const void* k, const void* v, void* o, float* lse,
              const flash_attention_fwd_fused_tiling_data* t, uint32_t kv_heads, cudaStream_t stream) {
    constexpr uint32_t kSmemBytes = Geom<HD, HDV>::kSmemBytes;
    static std::once_flag reg_once;
    std::call_once(reg_once, [] { register_error_word(read_error_word); });
    const uint64_t BH = static_cast<uint64_t>(t->B) * t->H;
    CUtensorMap tmq, tmk, tmv;
    const CUtensorMapDataType dt = kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const uint32_t box[3] = {64, 128, 1};
    {
        uint64_t dims[3] = {HD, t->S_q, BH};
        uint64_t strides[2] = {HD * 2, static_cast<uint64_t>(t->S_q) * HD * 2};
        int rc = encode_tmap(&tmq, dt, 3, q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    {
        uint64_t dims[3] = {HD, t->S_k, static_cast<uint64_t>(t->B) * kv_heads};
        uint64_t strides[2] = {HD * 2, static_cast<uint64_t>(t->S_k) * HD * 2};
        int rc = encode_tmap(&tmk, dt, 3, k, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
        uint64_t dims_v[3] = {HDV, t->S_k, static_cast<uint64_t>(t->B) * kv_heads};
        uint64_t strides_v[2] = {HDV * 2, static_cast<uint64_t>(t->S_k) * HDV * 2};
        rc = encode_tmap(&tmv, dt, 3, v, dims_v, strides_v, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    Params prm;
    prm.o = o;
    prm.lse = lse;
    prm.S_q = t->S_q;
    prm.S_k = t->S_k;
    prm.BH = static_cast<uint32_t>(BH);
    prm.group = t->H / kv_heads;
    prm.n_qblk = (t->S_q + 2 * kBM - 1) / (2 * kBM);
    const uint64_t pairs = BH * ((prm.n_qblk + 1) / 2);
    if (BH * prm.n_qblk > 0xffffffffull) return fail(HC_ERR_UNSUPPORTED, "flash_attention: too many work units");
    prm.num_pairs = static_cast<uint32_t>(pairs);
    prm.scale_log2 = t->scale * 1.4426950408889634f;
    prm.causal = t->maskType;
    if (int rc = set_max_dynamic_smem(reinterpret_cast<const void*>(fa_fwd_tc_kernel<kBF16, HD, HDV>), kSmemBytes,
                                      "fa_fwd_tc_kernel"))
        return rc;
    uint32_t grid = static_cast<uint32_t>(sm_count());
    if (grid > prm.num_pairs) grid = prm.num_pairs;
    fa_fwd_tc_kernel<kBF16, HD, HDV><<<grid, kThreads, kSmemBytes, stream>>>(tmq, tmk, tmv, prm);
    t_last_path = 1;
    return check_launch("fa_fwd_tc_kernel");
}

// The tensor-core kernel for the (D, D_v) pair: each of 64 and 128.
template <bool kBF16>
int launch_tc_dims(const void* q, const void* k, const void* v, void* o, float* lse,
                   const flash_attention_fwd_fused_tiling_data* t, uint32_t kv_heads, cudaStream_t stream) {
    if (t->D == 128 && t->D_v == 128) return launch_tc<kBF16, 128, 128>(q, k, v, o, lse, t, kv_heads, stream);
    if (t->D == 64 && t->D_v == 64) return launch_tc<kBF16, 64, 64>(q, k, v, o, lse, t, kv_heads, stream);
    if (t->D == 128) return launch_tc<kBF16, 128, 64>(q, k, v, o, lse, t, kv_heads, stream);
    return launch_tc<kBF16, 64, 128>(q, k, v, o, lse, t, kv_heads, stream);
}

template <typename T>
int launch_simt(const void* q, const void* k, const void* v, void* o, float* lse,
                const flash_attention_fwd_fused_tiling_data* t, uint32_t kv_heads, cudaStream_t stream) {
    const uint64_t rows = static_cast<uint64_t>(t->B) * t->H * t->S_q;
    uint64_t blocks = (rows + 7) / 8;
    const uint64_t cap = static_cast<uint64_t>(resident_blocks(reinterpret_cast<const void*>(fa_fwd_simt_kernel<T>), 256, 0));
    if (blocks > cap) blocks = cap;
    fa_fwd_simt_kernel<T><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
        static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(v), static_cast<T*>(o), lse,
        t->B * t->H, t->S_q, t->S_k, t->D, t->D_v, t->scale, t->maskType, t->H / kv_heads);
    t_last_path = 2;
    return check_launch("fa_fwd_simt_kernel");
}

}  // namespace fa
}  // namespace hc

using namespace hc;

namespace hc {
int fa_check_tiling(const flash_attention_fwd_fused_tiling_data* t, uint32_t kv_heads, int dtype) {
    if (!t) return fail(HC_ERR_INVALID, "flash_attention: null tiling");
    if (t->B == 0 || t->H == 0 || t->S_q == 0) return ok();
    if (kv_heads == 0 || t->H % kv_heads != 0)
        return fail(HC_ERR_INVALID, "flash_attention: kv_heads %u must divide H %u", kv_heads, t->H);
    if (t->S_k == 0) return fail(HC_ERR_INVALID, "flash_attention: S_k must be >= 1");
    if (t->D == 0 || t->D_v == 0 || t->D > 256 || t->D_v > 256)
        return fail(HC_ERR_UNSUPPORTED, "flash_attention: D=%u D_v=%u (1..256 supported)", t->D, t->D_v);
    if (t->maskType > 1) return fail(HC_ERR_INVALID, "flash_attention: maskType %u (0 none, 1 causal)", t->maskType);
    if (!std::isfinite(t->scale)) return fail(HC_ERR_INVALID, "flash_attention: scale must be finite");
    if (dtype != HC_DTYPE_BF16 && dtype != HC_DTYPE_F16 && dtype != HC_DTYPE_F32)
        return fail(HC_ERR_UNSUPPORTED, "flash_attention: dtype %d not supported (BF16, F16, F32)", dtype);
    return ok();
}
}  // namespace hc

extern "C" int hc_flash_attention_fwd_fused_gqa_launch(const void* q, const void* k, const void* v, void* o,
                                                       float* lse, const flash_attention_fwd_fused_tiling_data* t,
                                                       uint32_t kv_heads, int dtype, void* stream) {
    if (int rc = fa_check_tiling(t, kv_heads, dtype)) return rc;
    if (t->B == 0 || t->H == 0 || t->S_q == 0) return ok();
    if (!q || !k || !v || !o) return fail(HC_ERR_INVALID, "flash_attention: null pointer");
    if (fault_hit("launch")) return fail(HC_ERR_INJECTED, "flash_attention: injected launch failure");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool tc_shape = (t->D == 128 || t->D == 64) && (t->D_v == 128 || t->D_v == 64) && t->scale > 0.f &&
                          aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o);
    if (dtype == HC_DTYPE_BF16) {
        if (tc_shape) return fa::launch_tc_dims<true>(q, k, v, o, lse, t, kv_heads, s);
        return fa::launch_simt<bf16_t>(q, k, v, o, lse, t, kv_heads, s);
    }
    if (dtype == HC_DTYPE_F16) {
        if (tc_shape) return fa::launch_tc_dims<false>(q, k, v, o, lse, t, kv_heads, s);
        return fa::launch_simt<f16_t>(q, k, v, o, lse, t, kv_heads, s);
    }
    if (dtype == HC_DTYPE_F32) return fa::launch_simt<float>(q, k, v, o, lse, t, kv_heads, s);
    return fail(HC_ERR_UNSUPPORTED, "flash_attention: dtype %d not supported (BF16, F16, F32)", dtype);
}

extern "C" int hc_flash_attention_fwd_fused_launch(const void* q, const void* k, const void* v, void* o, float* lse,
                                                   const flash_attention_fwd_fused_tiling_data* t, int dtype,
                                                   void* stream) {
    return hc_flash_attention_fwd_fused_gqa_launch(q, k, v, o, lse, t, t ? t->H : 1u, dtype, stream);
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
