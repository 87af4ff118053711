// matmul_bias on B200: C = A . B + bias, fp32 accumulation.
//
// Follows the reference golden ops/matmul_bias/golden/matmul_bias_golden.cpp:6-27
// (C[m,n] = float(sum_k A[m,k] B[k,n]) + bias[n], bias optional), with bf16/fp16 operands
// and a single rounding of the fp32 result to the output type.
//
// Tensor-core path (bf16/fp16, K and N multiples of 8): persistent CTAs, 128x256 output tiles,
// 64-deep K blocks.
//   * warp 0 streams A (K-major, 128x64 panel) and B (MN-major, four 64x64 panels) into a
//     4-stage shared-memory ring with TMA (128-byte swizzle, no multicast);
//   * warp 1 (one thread) issues tcgen05.mma M=128 N=256 K=16 into one of two TMEM accumulators
//     (2 x 256 columns), so the epilogue of tile t overlaps the main loop of tile t+1;
//   * warps 2-5 drain the accumulator with tcgen05.ld (thread = row), add the bias, round and
//     store.
// Tiles are rasterised in groups of 16 M-tiles so that the CTAs in flight share A and B panels
// in L2.  Waits are bounded as in the attention kernel.
//
// SIMT path: fp32, or shapes whose rows are not 16-byte multiples.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <mutex>

#include "hc_device.cuh"
#include "hc_internal.h"
#include "sm100.cuh"
#include "tmap.h"

namespace hc {
namespace mm {

using namespace sm100;

constexpr uint32_t kBM = 128, kBN = 256, kBK = 64;
constexpr uint32_t kStages = 4;
constexpr uint32_t kThreads = 192;
constexpr uint32_t kABytes = kBM * kBK * 2;      // 16 KB
constexpr uint32_t kBPanel = kBK * 64 * 2;       // 8 KB: 64 k-rows x 64 n
constexpr uint32_t kBBytes = kBPanel * (kBN / 64);  // 32 KB
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr uint32_t kOffBar = kStages * kStageBytes;
constexpr uint32_t kSmemBytes = kOffBar + 256 + 1024;
constexpr uint32_t kGroupM = 16;

enum : uint32_t {
    kErrProducer = 1u << 0,
    kErrMmaFull = 1u << 1,
    kErrMmaAcc = 1u << 2,
    kErrEpi = 1u << 3,
    kErrDrain = 1u << 4,
};

__device__ uint32_t g_mm_error_word;

struct Params {
    void* c;
    const void* bias;
    uint32_t M, N, K, tiles_m, tiles_n, num_tiles, k_blocks;
};

struct Bars {
    uint64_t full[kStages], empty[kStages];
    uint64_t acc_full[2], acc_empty[2];
    uint64_t mma_done;
};

__device__ __forceinline__ void tile_coords(const Params& p, uint32_t t, uint32_t& tm, uint32_t& tn) {
    const uint32_t per_group = kGroupM * p.tiles_n;
    const uint32_t g = t / per_group;
    const uint32_t first_m = g * kGroupM;
    const uint32_t gsize = min(kGroupM, p.tiles_m - first_m);
    const uint32_t r = t - g * per_group;
    tm = first_m + r % gsize;
    tn = r / gsize;
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
__device__ __forceinline__ float to_f(uint16_t bits) {
    if (kBF16) return __uint_as_float(static_cast<uint32_t>(bits) << 16);
    return __half2float(*reinterpret_cast<const __half*>(&bits));
}

template <bool kBF16>
__global__ void __launch_bounds__(kThreads, 1)
    mm_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b, const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffBar + sizeof(Bars));
    volatile uint32_t* abort_flag = tmem_slot + 1;
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < kStages; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars->acc_full[b], 1);
            mbar_init(&bars->acc_empty[b], 128);
        }
        mbar_init(&bars->mma_done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tm_a);
        prefetch_tmap(&tm_b);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const uint32_t s_base = smem_u32(smem);

    if (warp == 0) {
        // ================================ TMA producer ================================
        if (lane == 0) {
            uint32_t stage = 0, phase = 0;
            int32_t pending[kStages];
            for (uint32_t s = 0; s < kStages; ++s) pending[s] = -1;
            bool ok = true;
            for (uint32_t t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
                uint32_t tm, tn;
                tile_coords(p, t, tm, tn);
                for (uint32_t kb = 0; kb < p.k_blocks; ++kb) {
                    if (!mbar_wait_bounded(&bars->empty[stage], phase ^ 1, abort_flag, &g_mm_error_word, kErrProducer)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = smem + stage * kStageBytes;
                    mbar_arrive_expect_tx(&bars->full[stage], kStageBytes);
                    tma_load_2d(st, &tm_a, &bars->full[stage], static_cast<int32_t>(kb * kBK),
                                static_cast<int32_t>(tm * kBM));
#pragma unroll
                    for (uint32_t pn = 0; pn < kBN / 64; ++pn)
                        tma_load_2d(st + kABytes + pn * kBPanel, &tm_b, &bars->full[stage],
                                    static_cast<int32_t>(tn * kBN + pn * 64), static_cast<int32_t>(kb * kBK));
                    pending[stage] = static_cast<int32_t>(phase);
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (!ok) {
                volatile uint32_t never = 0;
                for (uint32_t s = 0; s < kStages; ++s)
                    if (pending[s] >= 0)
                        mbar_wait_bounded(&bars->full[s], static_cast<uint32_t>(pending[s]), &never, &g_mm_error_word,
                                          kErrDrain, 1000000000ull);
            }
        }
    } else if (warp == 1) {
        // ================================= MMA issuer =================================
        if (lane == 0) {
            const uint32_t idesc = make_idesc_f16(kBF16, kBM, kBN, false, true);
            uint32_t stage = 0, phase = 0;
            bool ok = true;
            uint32_t it = 0;
            for (uint32_t t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x, ++it) {
                const uint32_t ab = it & 1;
                if (!mbar_wait_bounded(&bars->acc_empty[ab], ((it >> 1) & 1) ^ 1, abort_flag, &g_mm_error_word,
                                       kErrMmaAcc)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + ab * kBN;
                for (uint32_t kb = 0; kb < p.k_blocks; ++kb) {
                    if (!mbar_wait_bounded(&bars->full[stage], phase, abort_flag, &g_mm_error_word, kErrMmaFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = s_base + stage * kStageBytes;
                    const uint32_t b_addr = a_addr + kABytes;
#pragma unroll
                    for (uint32_t kk = 0; kk < kBK / 16; ++kk) {
                        uint64_t ad = make_sw128_desc(a_addr + kk * 32, 16, 1024);
                        uint64_t bd = make_sw128_desc(b_addr + kk * 2048, kBPanel, 1024);
                        mma_ss(d_tmem, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
                    }
                    tc_commit(&bars->empty[stage]);
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                tc_commit(&bars->acc_full[ab]);
            }
            tc_commit(&bars->mma_done);
            volatile uint32_t never = 0;
            mbar_wait_bounded(&bars->mma_done, 0, &never, &g_mm_error_word, kErrDrain, 1000000000ull);
        }
    } else {
        // ================================== epilogue ==================================
        const uint32_t quarter = warp & 3;  // warps 2,3,4,5 -> TMEM lane quarters 2,3,0,1
        const uint32_t r_local = quarter * 32 + lane;
        const uint32_t lane_field = (quarter * 32) << 16;
        uint32_t it = 0;
        for (uint32_t t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++it) {
            uint32_t tm, tn;
            tile_coords(p, t, tm, tn);
            const uint32_t ab = it & 1;
            bool ok = mbar_wait_bounded(&bars->acc_full[ab], (it >> 1) & 1, abort_flag, &g_mm_error_word, kErrEpi);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            const uint32_t row = tm * kBM + r_local;
            const uint32_t col0 = tn * kBN;
            const bool row_ok = row < p.M;
            uint16_t* crow = static_cast<uint16_t*>(p.c) + static_cast<size_t>(row) * p.N;
            const uint16_t* bias = static_cast<const uint16_t*>(p.bias);
#pragma unroll 1
            for (uint32_t c = 0; c < kBN / 32; ++c) {
                uint32_t acc[32];
                tmem_ld32(tmem_base + ab * kBN + c * 32 + lane_field, acc);
                tmem_wait_ld();
                const uint32_t n0 = col0 + c * 32;
                if (!row_ok || n0 >= p.N) continue;
                float v[32];
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    v[e] = __uint_as_float(acc[e]);
                    if (bias) {
                        uint32_t n = n0 + e;
                        v[e] = __fadd_rn(v[e], n < p.N ? to_f<kBF16>(bias[n]) : 0.f);
                    }
                }
                if (n0 + 32 <= p.N) {
                    uint4* dst = reinterpret_cast<uint4*>(crow + n0);  // N % 8 == 0 keeps 16 B alignment
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        dst[q] = make_uint4(pack2<kBF16>(v[8 * q + 0], v[8 * q + 1]), pack2<kBF16>(v[8 * q + 2], v[8 * q + 3]),
                                            pack2<kBF16>(v[8 * q + 4], v[8 * q + 5]), pack2<kBF16>(v[8 * q + 6], v[8 * q + 7]));
                } else {
                    for (uint32_t e = 0; e < 32 && n0 + e < p.N; ++e) {
                        uint32_t pk = pack2<kBF16>(v[e], 0.f);
                        crow[n0 + e] = static_cast<uint16_t>(pk & 0xffffu);
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&bars->acc_empty[ab]);
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        tmem_dealloc(tmem_base, 512);
    }
}

// ======================================================================================
// CTA-pair path (M >= 256): a cluster of two CTAs on two SMs computes 256x256 output tiles with
// tcgen05.mma cta_group::2 (M=256, N=256, K=16).  CTA rank r stages rows [128 r, 128 r + 128)
// of the A panel and columns [128 r, 128 r + 128) of the B panel (32 KB per 64-deep K block, a
// 6-stage ring); the even CTA's thread issues the MMAs, which read A from each CTA and both B
// halves, and accumulate each CTA's 128 rows x 256 columns in its own TMEM (two accumulators of
// 256 columns, so the epilogue overlaps the next tile).  Per output element this moves a third
// less operand data from L2 into shared memory than the 128x256 single-CTA tile.
//   * both producers' TMA loads complete on the even CTA's `full` barrier (whose expected byte
//     count covers both halves); the MMA commit releases the stage in both CTAs (CTA mask 0b11);
//   * each CTA's epilogue drains its own TMEM and arrives (one lane per warp) on the even CTA's
//     `acc_empty` barrier, which expects 4 warps x 2 CTAs.
// No TMA load multicasts.  Waits are bounded as in the single-CTA kernel; on an error each CTA
// unwinds, the even CTA drains the stages it armed, the odd CTA pauses 2 ms for its last copies
// (it cannot observe their completion), and the pair meets at a cluster barrier before TMEM is
// freed.
// ======================================================================================
constexpr uint32_t kStages2 = 6;
constexpr uint32_t kBHalf2 = kBPanel * 2;                // 16 KB: this CTA's 128 of the 256 B columns
constexpr uint32_t kStageBytes2 = kABytes + kBHalf2;     // 32 KB
constexpr uint32_t kOffBar2 = kStages2 * kStageBytes2;
constexpr uint32_t kSmemBytes2 = kOffBar2 + 256 + 1024;
constexpr uint32_t kGroupM2 = 8;                         // pair-tile rows per rasterisation group

struct Bars2 {
    uint64_t full[kStages2], empty[kStages2];
    uint64_t acc_full[2], acc_empty[2];
    uint64_t mma_done;
};

__device__ __forceinline__ void pair_tile_coords(const Params& p, uint32_t t, uint32_t& tm, uint32_t& tn) {
    const uint32_t per_group = kGroupM2 * p.tiles_n;
    const uint32_t g = t / per_group;
    const uint32_t first_m = g * kGroupM2;
    const uint32_t gsize = min(kGroupM2, p.tiles_m - first_m);
    const uint32_t r = t - g * per_group;
    tm = first_m + r % gsize;
    tn = r / gsize;
}

template <bool kBF16>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    mm_tc2_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b, const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Bars2* bars = reinterpret_cast<Bars2*>(smem + kOffBar2);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffBar2 + sizeof(Bars2));
    volatile uint32_t* abort_flag = tmem_slot + 1;
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();  // 0: issues the MMAs of the pair
    const uint32_t cluster = blockIdx.x / 2, clusters = gridDim.x / 2;  // p.tiles_m counts 256-row pair tiles

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < kStages2; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars->acc_full[b], 1);
            mbar_init(&bars->acc_empty[b], 8);
        }
        mbar_init(&bars->mma_done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, 512);
        tmem_relinquish_pair();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tm_a);
        prefetch_tmap(&tm_b);
    }
    tc_fence_before();
    cluster_sync_all();  // both CTAs' barriers are initialised before either signals the other
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const uint32_t s_base = smem_u32(smem);

    if (warp == 0) {
        // ================================ TMA producers ================================
        if (lane == 0) {
            uint32_t stage = 0, phase = 0;
            int32_t pending[kStages2];
            for (uint32_t s = 0; s < kStages2; ++s) pending[s] = -1;
            bool ok = true, issued = false;
            for (uint32_t t = cluster; t < p.num_tiles && ok; t += clusters) {
                uint32_t tm, tn;
                pair_tile_coords(p, t, tm, tn);
                for (uint32_t kb = 0; kb < p.k_blocks; ++kb) {
                    if (!mbar_wait_bounded(&bars->empty[stage], phase ^ 1, abort_flag, &g_mm_error_word, kErrProducer)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = smem + stage * kStageBytes2;
                    const uint32_t full_even = mapa_shared(smem_u32(&bars->full[stage]), 0);
                    if (rank == 0) mbar_arrive_expect_tx(&bars->full[stage], 2 * kStageBytes2);
                    tma_load_2d_pair(st, &tm_a, full_even, static_cast<int32_t>(kb * kBK),
                                     static_cast<int32_t>(tm * 2 * kBM + rank * kBM));
#pragma unroll
                    for (uint32_t pn = 0; pn < 2; ++pn)
                        tma_load_2d_pair(st + kABytes + pn * kBPanel, &tm_b, full_even,
                                         static_cast<int32_t>(tn * kBN + rank * 128 + pn * 64),
                                         static_cast<int32_t>(kb * kBK));
                    issued = true;
                    pending[stage] = static_cast<int32_t>(phase);
                    if (++stage == kStages2) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (!ok) {
                if (rank == 0) {
                    volatile uint32_t never = 0;
                    for (uint32_t s = 0; s < kStages2; ++s)
                        if (pending[s] >= 0)
                            mbar_wait_bounded(&bars->full[s], static_cast<uint32_t>(pending[s]), &never,
                                              &g_mm_error_word, kErrDrain, 1000000000ull);
                } else if (issued) {
                    spin_ns(2000000ull);
                }
            }
        }
    } else if (warp == 1) {
        // ====================== MMA issuer (even CTA, for the pair) =====================
        if (rank == 0 && lane == 0) {
            const uint32_t idesc = make_idesc_f16(kBF16, 2 * kBM, kBN, false, true);
            uint32_t stage = 0, phase = 0;
            bool ok = true;
            uint32_t it = 0;
            for (uint32_t t = cluster; t < p.num_tiles && ok; t += clusters, ++it) {
                const uint32_t ab = it & 1;
                if (!mbar_wait_bounded_cluster(&bars->acc_empty[ab], ((it >> 1) & 1) ^ 1, abort_flag, &g_mm_error_word,
                                               kErrMmaAcc)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + ab * kBN;
                for (uint32_t kb = 0; kb < p.k_blocks; ++kb) {
                    if (!mbar_wait_bounded_cluster(&bars->full[stage], phase, abort_flag, &g_mm_error_word,
                                                   kErrMmaFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = s_base + stage * kStageBytes2;
                    const uint32_t b_addr = a_addr + kABytes;
#pragma unroll
                    for (uint32_t kk = 0; kk < kBK / 16; ++kk) {
                        const uint64_t ad = make_sw128_desc(a_addr + kk * 32, 16, 1024);
                        const uint64_t bd = make_sw128_desc(b_addr + kk * 2048, kBPanel, 1024);
                        mma_ss_pair(d_tmem, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
                    }
                    tc_commit_pair(&bars->empty[stage], 0x3);
                    if (++stage == kStages2) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                tc_commit_pair(&bars->acc_full[ab], 0x3);
            }
            // All issued MMAs complete before TMEM is freed (normal and error paths alike).
            tc_commit_pair(&bars->mma_done, 0x1);
            volatile uint32_t never = 0;
            mbar_wait_bounded(&bars->mma_done, 0, &never, &g_mm_error_word, kErrDrain, 1000000000ull);
        }
    } else {
        // ================================== epilogues ==================================
        const uint32_t quarter = warp & 3;  // warps 2,3,4,5 -> TMEM lane quarters 2,3,0,1
        const uint32_t r_local = quarter * 32 + lane;
        const uint32_t lane_field = (quarter * 32) << 16;
        uint32_t it = 0;
        for (uint32_t t = cluster; t < p.num_tiles; t += clusters, ++it) {
            uint32_t tm, tn;
            pair_tile_coords(p, t, tm, tn);
            const uint32_t ab = it & 1;
            bool ok = mbar_wait_bounded_cluster(&bars->acc_full[ab], (it >> 1) & 1, abort_flag, &g_mm_error_word,
                                                kErrEpi);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            const uint32_t row = tm * 2 * kBM + rank * kBM + r_local;
            const uint32_t col0 = tn * kBN;
            const bool row_ok = row < p.M;
            uint16_t* crow = static_cast<uint16_t*>(p.c) + static_cast<size_t>(row) * p.N;
            const uint16_t* bias = static_cast<const uint16_t*>(p.bias);
#pragma unroll 1
            for (uint32_t c = 0; c < kBN / 32; ++c) {
                uint32_t acc[32];
                tmem_ld32(tmem_base + ab * kBN + c * 32 + lane_field, acc);
                tmem_wait_ld();
                const uint32_t n0 = col0 + c * 32;
                if (!row_ok || n0 >= p.N) continue;
                float v[32];
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    v[e] = __uint_as_float(acc[e]);
                    if (bias) {
                        uint32_t n = n0 + e;
                        v[e] = __fadd_rn(v[e], n < p.N ? to_f<kBF16>(bias[n]) : 0.f);
                    }
                }
                if (n0 + 32 <= p.N) {
                    uint4* dst = reinterpret_cast<uint4*>(crow + n0);  // N % 8 == 0 keeps 16 B alignment
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        dst[q] = make_uint4(pack2<kBF16>(v[8 * q + 0], v[8 * q + 1]), pack2<kBF16>(v[8 * q + 2], v[8 * q + 3]),
                                            pack2<kBF16>(v[8 * q + 4], v[8 * q + 5]), pack2<kBF16>(v[8 * q + 6], v[8 * q + 7]));
                } else {
                    for (uint32_t e = 0; e < 32 && n0 + e < p.N; ++e) {
                        uint32_t pk = pack2<kBF16>(v[e], 0.f);
                        crow[n0 + e] = static_cast<uint16_t>(pk & 0xffffu);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&bars->acc_empty[ab]), 0));
        }
    }

    tc_fence_before();
    __syncwarp();
    cluster_sync_all();  // neither CTA frees TMEM or exits while the pair still uses its memory
    tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        tmem_dealloc_pair(tmem_base, 512);
    }
}

// ======================================================================================
// SIMT fallback: 64x64 output tiles, 16x16 threads, 4x4 outputs per thread, fp32 math.
// ======================================================================================
template <typename T>
__global__ void __launch_bounds__(256) mm_simt_kernel(const T* __restrict__ A, const T* __restrict__ B,
                                                      const T* __restrict__ bias, T* __restrict__ C, uint32_t M,
                                                      uint32_t N, uint32_t K) {
    __shared__ float As[16][64 + 1];
    __shared__ float Bs[16][64 + 1];
    const uint32_t tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const uint32_t m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
    float acc[4][4] = {};
    for (uint32_t k0 = 0; k0 < K; k0 += 16) {
        for (uint32_t i = threadIdx.x; i < 16 * 64; i += 256) {
            uint32_t kk = i % 16, mm = i / 16;
            uint32_t gm = m0 + mm, gk = k0 + kk;
            As[kk][mm] = (gm < M && gk < K) ? elem<T>::to_f(A[static_cast<size_t>(gm) * K + gk]) : 0.f;
            uint32_t nn = i % 64, kb = i / 64;
            uint32_t gn = n0 + nn, gk2 = k0 + kb;
            Bs[kb][nn] = (gn < N && gk2 < K) ? elem<T>::to_f(B[static_cast<size_t>(gk2) * N + gn]) : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint32_t gm = m0 + ty * 4 + i;
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint32_t gn = n0 + tx * 4 + j;
            if (gn >= N) continue;
            float v = acc[i][j];
            if (bias) v = __fadd_rn(v, elem<T>::to_f(bias[gn]));
            C[static_cast<size_t>(gm) * N + gn] = elem<T>::from_f(v);
        }
    }
}

uint32_t read_error_word(const char** name) {
    *name = "matmul_bias";
    uint32_t word = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&word, g_mm_error_word, sizeof(word)) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (word) cudaMemcpyToSymbol(g_mm_error_word, &zero, sizeof(zero));
    return word;
}

thread_local int t_last_path = 0;

// CTA pairs of the pair kernel that fit on the current device at once (one pair per two SMs),
// cached per device.
int pair_clusters() {
    static std::mutex mu;
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return 0;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (cache[dev] == 0) {
        int n = sm_count() / 2;
        if (set_max_dynamic_smem(reinterpret_cast<const void*>(mm_tc2_kernel<true>), kSmemBytes2, "mm_tc2_kernel") ==
            HC_OK) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(2 * n);
            cfg.blockDim = dim3(kThreads);
            cfg.dynamicSmemBytes = kSmemBytes2;
            int active = 0;
            if (cudaOccupancyMaxActiveClusters(&active, mm_tc2_kernel<true>, &cfg) == cudaSuccess && active > 0)
                n = active < n ? active : n;
            else
                cudaGetLastError();
        }
        cache[dev] = n > 0 ? n : -1;
    }
    return cache[dev] > 0 ? cache[dev] : 0;
}

template <bool kBF16>
int launch_tc(const void* A, const void* B, const void* bias, void* C, const matmul_bias_tiling_data* t,
              cudaStream_t stream) {
    static std::once_flag reg_once;
    std::call_once(reg_once, [] { register_error_word(read_error_word); });
    const CUtensorMapDataType dt = kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUtensorMap tma, tmb;
    {
        uint64_t dims[2] = {t->K, t->M};
        uint64_t strides[1] = {static_cast<uint64_t>(t->K) * 2};
        uint32_t box[2] = {kBK, kBM};
        int rc = encode_tmap(&tma, dt, 2, A, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    {
        uint64_t dims[2] = {t->N, t->K};
        uint64_t strides[1] = {static_cast<uint64_t>(t->N) * 2};
        uint32_t box[2] = {64, kBK};
        int rc = encode_tmap(&tmb, dt, 2, B, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    }
    Params prm;
    prm.c = C;
    prm.bias = bias;
    prm.M = t->M;
    prm.N = t->N;
    prm.K = t->K;
    prm.tiles_m = (t->M + kBM - 1) / kBM;
    prm.tiles_n = (t->N + kBN - 1) / kBN;
    prm.num_tiles = prm.tiles_m * prm.tiles_n;
    prm.k_blocks = (t->K + kBK - 1) / kBK;
    if (t->M >= 2 * kBM && pair_clusters() > 0) {
        // CTA pairs: tiles_m counts 256-row pair tiles
        prm.tiles_m = (t->M + 2 * kBM - 1) / (2 * kBM);
        prm.num_tiles = prm.tiles_m * prm.tiles_n;
        if (int rc = set_max_dynamic_smem(reinterpret_cast<const void*>(mm_tc2_kernel<kBF16>), kSmemBytes2,
                                          "mm_tc2_kernel"))
            return rc;
        uint32_t clusters = static_cast<uint32_t>(pair_clusters());
        if (clusters > prm.num_tiles) clusters = prm.num_tiles;
        mm_tc2_kernel<kBF16><<<2 * clusters, kThreads, kSmemBytes2, stream>>>(tma, tmb, prm);
        t_last_path = 3;
        return check_launch("mm_tc2_kernel");
    }
    if (int rc = set_max_dynamic_smem(reinterpret_cast<const void*>(mm_tc_kernel<kBF16>), kSmemBytes, "mm_tc_kernel"))
        return rc;
    uint32_t grid = static_cast<uint32_t>(sm_count());
    if (grid > prm.num_tiles) grid = prm.num_tiles;
    mm_tc_kernel<kBF16><<<grid, kThreads, kSmemBytes, stream>>>(tma, tmb, prm);
    t_last_path = 1;
    return check_launch("mm_tc_kernel");
}

template <typename T>
int launch_simt(const void* A, const void* B, const void* bias, void* C, const matmul_bias_tiling_data* t,
                cudaStream_t stream) {
    dim3 grid((t->N + 63) / 64, (t->M + 63) / 64);
    if (grid.y > 65535) return fail(HC_ERR_UNSUPPORTED, "matmul_bias SIMT path: M too large");
    mm_simt_kernel<T><<<grid, 256, 0, stream>>>(static_cast<const T*>(A), static_cast<const T*>(B),
                                                static_cast<const T*>(bias), static_cast<T*>(C), t->M, t->N, t->K);
    t_last_path = 2;
    return check_launch("mm_simt_kernel");
}

}  // namespace mm
}  // namespace hc

using namespace hc;

extern "C" int hc_matmul_bias_launch(const void* A, const void* B, const void* bias, void* C,
                                     const matmul_bias_tiling_data* t, int dtype, void* stream) {
    if (!t) return fail(HC_ERR_INVALID, "matmul_bias: null tiling");
    if (t->M == 0 || t->N == 0) return ok();
    if (!A || !B || !C) return fail(HC_ERR_INVALID, "matmul_bias: null pointer");
    if (t->K == 0) return fail(HC_ERR_INVALID, "matmul_bias: K must be >= 1");
    if (fault_hit("launch")) return fail(HC_ERR_INJECTED, "matmul_bias: injected launch failure");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool tc_shape = (t->K % 8 == 0) && (t->N % 8 == 0) && aligned16(A) && aligned16(B) && aligned16(C);
    switch (dtype) {
        case HC_DTYPE_BF16:
            return tc_shape ? mm::launch_tc<true>(A, B, bias, C, t, s) : mm::launch_simt<bf16_t>(A, B, bias, C, t, s);
        case HC_DTYPE_F16:
            return tc_shape ? mm::launch_tc<false>(A, B, bias, C, t, s) : mm::launch_simt<f16_t>(A, B, bias, C, t, s);
        case HC_DTYPE_F32: return mm::launch_simt<float>(A, B, bias, C, t, s);
        default: return fail(HC_ERR_UNSUPPORTED, "matmul_bias: dtype %d not supported", dtype);
    }
}

extern "C" int hc_matmul_bias_last_path(void) { return mm::t_last_path; }
