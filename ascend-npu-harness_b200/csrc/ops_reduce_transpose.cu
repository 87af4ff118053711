// reduce_sum_lastdim and transpose_2d_4d: HBM-bound reductions and index permutations.
//
// reduce_sum_lastdim follows ops/reduce_sum_lastdim/golden/reduce_sum_lastdim_golden.cpp:10-46
// (fp32 Kahan-compensated row sums); here each lane keeps a Kahan sum over its strided slice and
// the lanes' partial sums are combined by a shuffle tree.
// transpose_2d_4d follows ops/transpose_2d_4d/golden/transpose_2d_4d_golden.cpp:7-62; all three
// modes are batched 2-D transposes staged through shared-memory tiles, bit-exact by construction.
#include <cuda_runtime.h>

#include "hc_device.cuh"
#include "hc_internal.h"

namespace hc {
namespace {

// ---------------------------------------------------------------------------------------
// reduce_sum_lastdim
// ---------------------------------------------------------------------------------------
struct Kahan {
    float sum = 0.f, comp = 0.f;
    __device__ void add(float v) {
        float y = __fsub_rn(v, comp);
        float t = __fadd_rn(sum, y);
        comp = __fsub_rn(__fsub_rn(t, sum), y);
        sum = t;
    }
};

// One warp per row (rows of up to a few thousand elements).
template <typename T, bool kVec>
__global__ void __launch_bounds__(256) reduce_rows_warp_kernel(const T* __restrict__ x, float* __restrict__ out,
                                                               uint32_t rows, uint32_t K) {
    const uint32_t warps_total = gridDim.x * (blockDim.x / 32);
    const uint32_t lane = threadIdx.x & 31;
    for (uint32_t r = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; r < rows; r += warps_total) {
        const T* row = x + static_cast<size_t>(r) * K;
        Kahan acc;
        if (kVec) {
            constexpr int P = elem<T>::kPack;
            const pack<T>* pr = reinterpret_cast<const pack<T>*>(row);
            for (uint32_t i = lane; i < K / P; i += 32) {
                pack<T> v = ld_stream(pr + i);
#pragma unroll
                for (int e = 0; e < P; ++e) acc.add(elem<T>::to_f(v.v[e]));
            }
        } else {
            for (uint32_t k = lane; k < K; k += 32) acc.add(elem<T>::to_f(row[k]));
        }
        float s = warp_sum(acc.sum - acc.comp);
        if (lane == 0) out[r] = s;
    }
}

// One block of 256 threads per row (long rows).
template <typename T, bool kVec>
__global__ void __launch_bounds__(256) reduce_rows_block_kernel(const T* __restrict__ x, float* __restrict__ out,
                                                                uint32_t rows, uint32_t K) {
    __shared__ float partial[8];
    for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const T* row = x + static_cast<size_t>(r) * K;
        Kahan acc;
        if (kVec) {
            constexpr int P = elem<T>::kPack;
            const pack<T>* pr = reinterpret_cast<const pack<T>*>(row);
            for (uint32_t i = threadIdx.x; i < K / P; i += blockDim.x) {
                pack<T> v = ld_stream(pr + i);
#pragma unroll
                for (int e = 0; e < P; ++e) acc.add(elem<T>::to_f(v.v[e]));
            }
        } else {
            for (uint32_t k = threadIdx.x; k < K; k += blockDim.x) acc.add(elem<T>::to_f(row[k]));
        }
        float s = warp_sum(acc.sum - acc.comp);
        if ((threadIdx.x & 31) == 0) partial[threadIdx.x / 32] = s;
        __syncthreads();
        if (threadIdx.x < 32) {
            float v = threadIdx.x < blockDim.x / 32 ? partial[threadIdx.x] : 0.f;
            v = warp_sum(v);
            if (threadIdx.x == 0) out[r] = v;
        }
        __syncthreads();
    }
}

template <typename T>
int launch_reduce(const void* x, float* out, uint32_t rows, uint32_t K, void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const T* tx = static_cast<const T*>(x);
    bool vec = aligned16(x) && (K % elem<T>::kPack == 0);
    if (K <= 8192) {
        int blocks = static_cast<int>((rows + 7) / 8);
        int cap = sm_count() * 8;
        if (blocks > cap) blocks = cap;
        if (vec) reduce_rows_warp_kernel<T, true><<<blocks, 256, 0, s>>>(tx, out, rows, K);
        else reduce_rows_warp_kernel<T, false><<<blocks, 256, 0, s>>>(tx, out, rows, K);
    } else {
        int blocks = static_cast<int>(rows);
        int cap = sm_count() * 8;
        if (blocks > cap) blocks = cap;
        if (vec) reduce_rows_block_kernel<T, true><<<blocks, 256, 0, s>>>(tx, out, rows, K);
        else reduce_rows_block_kernel<T, false><<<blocks, 256, 0, s>>>(tx, out, rows, K);
    }
    return check_launch("reduce_sum_lastdim");
}

// ---------------------------------------------------------------------------------------
// transpose: out[b][c][r] = in[b][r][c] for `batch` matrices of R x C elements.
// ---------------------------------------------------------------------------------------
constexpr int kTile = 32;
constexpr int kRowsPerPass = 8;

template <typename E>
__global__ void __launch_bounds__(kTile * kRowsPerPass) transpose_kernel(const E* __restrict__ in, E* __restrict__ out,
                                                                         uint32_t batch, uint32_t R, uint32_t C) {
    __shared__ E tile[kTile][kTile + 1];
    const uint64_t tiles_r = (R + kTile - 1) / kTile;
    const uint64_t tiles_c = (C + kTile - 1) / kTile;
    const uint64_t per_batch = tiles_r * tiles_c;
    const uint64_t total = per_batch * batch;
    const size_t mat = static_cast<size_t>(R) * C;
    for (uint64_t t = blockIdx.x; t < total; t += gridDim.x) {
        uint64_t b = t / per_batch;
        uint64_t rem = t % per_batch;
        uint32_t r0 = static_cast<uint32_t>(rem / tiles_c) * kTile;
        uint32_t c0 = static_cast<uint32_t>(rem % tiles_c) * kTile;
        const E* src = in + b * mat;
        E* dst = out + b * mat;
        // Read rows r0.. of the tile (coalesced along c).
        for (int i = threadIdx.y; i < kTile; i += kRowsPerPass) {
            uint32_t r = r0 + i, c = c0 + threadIdx.x;
            if (r < R && c < C) tile[i][threadIdx.x] = src[static_cast<size_t>(r) * C + c];
        }
        __syncthreads();
        // Write rows c0.. of the output (coalesced along r).
        for (int i = threadIdx.y; i < kTile; i += kRowsPerPass) {
            uint32_t c = c0 + i, r = r0 + threadIdx.x;
            if (r < R && c < C) dst[static_cast<size_t>(c) * R + r] = tile[threadIdx.x][i];
        }
        __syncthreads();
    }
}

// 2-byte elements: 64 x 64 tiles, so that every warp access is one 128-byte row segment (a 32 x 32
// tile of 2-byte elements would move 64-byte segments).  A lane moves two neighbouring elements
// as one 32-bit word (two 16-bit accesses where a word would be misaligned or cross the edge).
// Shared-memory rows are 65 elements long: the transposed reads (rows 2l and 2l+1 of one column)
// then fall on 32 different banks.
constexpr int kT16 = 64;

__global__ void __launch_bounds__(kTile * kRowsPerPass) transpose16_kernel(const uint16_t* __restrict__ in,
                                                                           uint16_t* __restrict__ out, uint32_t batch,
                                                                           uint32_t R, uint32_t C) {
    constexpr int kRowsPerThread = kT16 / kRowsPerPass;  // 8
    __shared__ uint16_t tile[kT16][kT16 + 1];
    const uint64_t tiles_r = (R + kT16 - 1) / kT16;
    const uint64_t tiles_c = (C + kT16 - 1) / kT16;
    const uint64_t per_batch = tiles_r * tiles_c;
    const uint64_t total = per_batch * batch;
    const size_t mat = static_cast<size_t>(R) * C;
    const uint32_t l2 = 2 * threadIdx.x;
    // The tile's rows r0+i (i = threadIdx.y + 8k) are fetched into registers one tile ahead, so
    // the loads of tile t+1 are in flight while tile t is written out.
    struct Coord {
        uint64_t b;
        uint32_t r0, c0;
    };
    auto coord = [&](uint64_t t) {
        const uint64_t rem = t % per_batch;
        return Coord{t / per_batch, static_cast<uint32_t>(rem / tiles_c) * kT16, static_cast<uint32_t>(rem % tiles_c) * kT16};
    };
    // A 32-bit access needs an even element offset from the 4-byte aligned buffer start: the
    // parity is that of the batch base b * mat plus the offset inside the matrix.
    auto fetch = [&](const Coord& k, uint32_t (&w)[kRowsPerThread]) {
        const uint16_t* src = in + k.b * mat;
        const size_t base_par = (k.b * mat) & 1;
#pragma unroll
        for (int q = 0; q < kRowsPerThread; ++q) {
            const uint32_t r = k.r0 + threadIdx.y + q * kRowsPerPass, c = k.c0 + l2;
            uint32_t v = 0;
            if (r < R) {
                const size_t o = static_cast<size_t>(r) * C + c;
                if (c + 1 < C && ((base_par + o) & 1) == 0) {
                    v = __ldcs(reinterpret_cast<const unsigned int*>(src + o));
                } else {
                    if (c < C) v = src[o];
                    if (c + 1 < C) v |= static_cast<uint32_t>(src[o + 1]) << 16;
                }
            }
            w[q] = v;
        }
    };
    uint32_t w[kRowsPerThread];
    uint64_t t = blockIdx.x;
    if (t < total) fetch(coord(t), w);
    for (; t < total; t += gridDim.x) {
        const Coord k = coord(t);
#pragma unroll
        for (int q = 0; q < kRowsPerThread; ++q) {
            const int i = threadIdx.y + q * kRowsPerPass;
            tile[i][l2] = static_cast<uint16_t>(w[q]);
            tile[i][l2 + 1] = static_cast<uint16_t>(w[q] >> 16);
        }
        __syncthreads();
        if (t + gridDim.x < total) fetch(coord(t + gridDim.x), w);
        // Rows c0.. of the output, two elements per lane.
        uint16_t* dst = out + k.b * mat;
        const size_t base_par = (k.b * mat) & 1;
#pragma unroll
        for (int q = 0; q < kRowsPerThread; ++q) {
            const int i = threadIdx.y + q * kRowsPerPass;
            const uint32_t c = k.c0 + i, r = k.r0 + l2;
            if (c >= C) continue;
            const size_t o = static_cast<size_t>(c) * R + r;
            const uint16_t lo = tile[l2][i], hi = tile[l2 + 1][i];
            if (r + 1 < R && ((base_par + o) & 1) == 0) {
                __stcs(reinterpret_cast<unsigned int*>(dst + o),
                       static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16));
            } else {
                if (r < R) dst[o] = lo;
                if (r + 1 < R) dst[o + 1] = hi;
            }
        }
        __syncthreads();
    }
}

int launch_transpose16(const void* src, void* dst, uint32_t batch, uint32_t R, uint32_t C, void* stream) {
    const uint64_t tiles = static_cast<uint64_t>((R + kT16 - 1) / kT16) * ((C + kT16 - 1) / kT16) * batch;
    const uint64_t cap = static_cast<uint64_t>(sm_count()) * 8;
    const int blocks = static_cast<int>(tiles < cap ? tiles : cap);
    if (blocks == 0) return ok();
    transpose16_kernel<<<blocks, dim3(kTile, kRowsPerPass), 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t*>(src), static_cast<uint16_t*>(dst), batch, R, C);
    return check_launch("transpose_2d_4d");
}

template <typename E>
int launch_transpose(const void* src, void* dst, uint32_t batch, uint32_t R, uint32_t C, void* stream) {
    uint64_t tiles = static_cast<uint64_t>((R + kTile - 1) / kTile) * ((C + kTile - 1) / kTile) * batch;
    uint64_t cap = static_cast<uint64_t>(sm_count()) * 8;
    int blocks = static_cast<int>(tiles < cap ? tiles : cap);
    if (blocks == 0) return ok();
    transpose_kernel<E><<<blocks, dim3(kTile, kRowsPerPass), 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const E*>(src), static_cast<E*>(dst), batch, R, C);
    return check_launch("transpose_2d_4d");
}

}  // namespace
}  // namespace hc

using namespace hc;

extern "C" int hc_reduce_sum_lastdim_launch(const void* x, float* out, const reduce_sum_lastdim_tiling_data* t, int dtype,
                                            void* stream) {
    if (!t) return fail(HC_ERR_INVALID, "reduce_sum_lastdim: null tiling");
    // Same checks as ops/reduce_sum_lastdim/golden/reduce_sum_lastdim_golden.cpp:13-18.
    if (!x || !out) return fail(HC_ERR_INVALID, "reduce_sum_lastdim: null pointer");
    if (t->totalRows == 0 || t->K == 0) return fail(HC_ERR_INVALID, "reduce_sum_lastdim: invalid dimensions");
    if (fault_hit("launch")) return fail(HC_ERR_INJECTED, "reduce_sum_lastdim: injected launch failure");
    switch (dtype) {
        case HC_DTYPE_F32: return launch_reduce<float>(x, out, t->totalRows, t->K, stream);
        case HC_DTYPE_F16: return launch_reduce<f16_t>(x, out, t->totalRows, t->K, stream);
        case HC_DTYPE_BF16: return launch_reduce<bf16_t>(x, out, t->totalRows, t->K, stream);
        default: return fail(HC_ERR_UNSUPPORTED, "reduce_sum_lastdim: dtype %d not supported", dtype);
    }
}

extern "C" int hc_transpose_2d_4d_launch(const void* src, void* dst, const transpose_2d_4d_tiling_data* t, int dtype,
                                         void* stream) {
    if (!t) return fail(HC_ERR_INVALID, "transpose_2d_4d: null tiling");
    if (!src || !dst) return fail(HC_ERR_INVALID, "transpose_2d_4d: null pointer");
    size_t es = dtype_size(dtype);
    if (es == 0) return fail(HC_ERR_UNSUPPORTED, "transpose_2d_4d: dtype %d unknown", dtype);
    uint32_t batch, R, C;
    if (t->mode == 0) {
        batch = 1; R = t->M; C = t->N_dim;
    } else if (t->mode == 1) {  // NCHW -> NHWC: per n, [C][H*W] -> [H*W][C]
        batch = t->M; R = t->N_dim; C = t->H * t->W;
    } else if (t->mode == 2) {  // NHWC -> NCHW: per n, [H*W][C] -> [C][H*W]
        batch = t->M; R = t->H * t->W; C = t->N_dim;
    } else {
        return fail(HC_ERR_INVALID, "transpose_2d_4d: mode %u (0 = 2D, 1 = NCHW->NHWC, 2 = NHWC->NCHW)", t->mode);
    }
    if (batch == 0 || R == 0 || C == 0) return ok();
    if (fault_hit("launch")) return fail(HC_ERR_INJECTED, "transpose_2d_4d: injected launch failure");
    switch (es) {
        case 1: return launch_transpose<uint8_t>(src, dst, batch, R, C, stream);
        case 2:
            if ((reinterpret_cast<uintptr_t>(src) & 3) == 0 && (reinterpret_cast<uintptr_t>(dst) & 3) == 0)
                return launch_transpose16(src, dst, batch, R, C, stream);
            return launch_transpose<uint16_t>(src, dst, batch, R, C, stream);
        default: return launch_transpose<uint32_t>(src, dst, batch, R, C, stream);
    }
}
