// reduce_sum_lastdim and transpose_2d_4d: HBM-bound reductions and index permutations.
//
// reduce_sum_lastdim follows ops/reduce_sum_lastdim/golden/reduce_sum_lastdim_golden.cpp:10-46
// (fp32 Kahan-compensated row sums); here each lane keeps a Kahan sum over its strided slice and
// the lanes' partial sums are combined by a shuffle tree.
// transpose_2d_4d follows ops/transpose_2d_4d/golden/transpose_2d_4d_golden.cpp:7-62; all three
// modes are batched 2-D transposes staged through shared-memory tiles, bit-exact by construction.
#include <cuda_runtime.h>

#include <mutex>

#include "hc_device.cuh"
#include "hc_internal.h"
#include "sm100.cuh"
#include "tmap.h"

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
        auto kernel = vec ? reduce_rows_warp_kernel<T, true> : reduce_rows_warp_kernel<T, false>;
        int blocks = static_cast<int>((rows + 7) / 8);
        const int cap = resident_blocks(reinterpret_cast<const void*>(kernel), 256, 0);
        if (blocks > cap) blocks = cap;
        kernel<<<blocks, 256, 0, s>>>(tx, out, rows, K);
    } else {
        auto kernel = vec ? reduce_rows_block_kernel<T, true> : reduce_rows_block_kernel<T, false>;
        int blocks = static_cast<int>(rows);
        const int cap = resident_blocks(reinterpret_cast<const void*>(kernel), 256, 0);
        if (blocks > cap) blocks = cap;
        kernel<<<blocks, 256, 0, s>>>(tx, out, rows, K);
    }
    return check_launch("reduce_sum_lastdim");
}

// ---------------------------------------------------------------------------------------
// transpose: out[b][c][r] = in[b][r][c] for `batch` matrices of R x C elements.
// ---------------------------------------------------------------------------------------
constexpr int kTile = 32;
constexpr int kRowsPerPass = 8;

// Tile index t -> (matrix b, first row r0, first column c0) with 32-bit multiply-shift divisions
// (the launchers keep the tile count below 2^32); a 64-bit division per tile costs more
// instructions than moving the tile.
struct TileMap {
    FastDiv per_batch, tiles_c;
    uint32_t total;
    size_t mat;
    __device__ __forceinline__ void at(uint32_t t, uint32_t tile_r, uint32_t tile_c, uint64_t& b, uint32_t& r0,
                                       uint32_t& c0) const {
        const uint32_t bb = per_batch.div(t);
        const uint32_t rem = t - bb * per_batch.d;
        const uint32_t tr = tiles_c.div(rem);
        b = bb;
        r0 = tr * tile_r;
        c0 = (rem - tr * tiles_c.d) * tile_c;
    }
};

// Fills `m` for `batch` matrices of R x C in tiles of tile_r rows x tile_c columns; false when the
// tile count does not fit 32 bits.
bool make_tile_map(TileMap& m, uint32_t batch, uint32_t R, uint32_t C, uint32_t tile_r, uint32_t tile_c) {
    const uint64_t tiles_r = (static_cast<uint64_t>(R) + tile_r - 1) / tile_r;
    const uint64_t tiles_c = (static_cast<uint64_t>(C) + tile_c - 1) / tile_c;
    const uint64_t total = tiles_r * tiles_c * batch;
    if (tiles_r * tiles_c >= (1ull << 32) || total >= (1ull << 32)) return false;
    m.per_batch.init(static_cast<uint32_t>(tiles_r * tiles_c));
    m.tiles_c.init(static_cast<uint32_t>(tiles_c));
    m.total = static_cast<uint32_t>(total);
    m.mat = static_cast<size_t>(R) * C;
    return true;
}

template <typename E>
__global__ void __launch_bounds__(kTile * kRowsPerPass) transpose_kernel(const E* __restrict__ in, E* __restrict__ out,
                                                                         uint32_t R, uint32_t C, TileMap map) {
    __shared__ E tile[kTile][kTile + 1];
    for (uint32_t t = blockIdx.x; t < map.total; t += gridDim.x) {
        uint64_t b;
        uint32_t r0, c0;
        map.at(t, kTile, kTile, b, r0, c0);
        const E* src = in + b * map.mat;
        E* dst = out + b * map.mat;
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

// 2-byte elements: 64 x 64 tiles moved as 2 x 2 blocks.  On the way in, lane x of row-pair p
// loads the 32-bit words (r, c..c+1) and (r+1, c..c+1), r = r0 + 2p, c = c0 + 2x; two byte
// permutes turn them into the output words (c, r..r+1) and (c+1, r..r+1), which go to shared
// memory as blk[h][x][p].  On the way out, lane x writes output word (c0 + 2q + h, r0 + 2x) from
// blk[h][q][x].  Every warp access is a 128-byte row segment, and with rows of 33 words both
// shared-memory phases touch 32 different banks.  Words that would be misaligned, or that cross
// the matrix edge, are moved as two 16-bit accesses.
constexpr int kT16 = 64;

__global__ void __launch_bounds__(kTile * kRowsPerPass) transpose16_kernel(const uint16_t* __restrict__ in,
                                                                           uint16_t* __restrict__ out, uint32_t R,
                                                                           uint32_t C, TileMap map) {
    constexpr int kPairsPerThread = kT16 / 2 / kRowsPerPass;  // 4 row pairs = 8 loaded words
    constexpr int kOutPerThread = kT16 / kRowsPerPass;         // 8 output words
    __shared__ uint32_t blk[2][kT16 / 2][kT16 / 2 + 1];
    const uint32_t lx = threadIdx.x, ly = threadIdx.y;
    // A 32-bit access needs an even element offset from the 4-byte aligned buffer start: the
    // parity is that of the batch base b * mat plus the offset inside the matrix.
    auto load_word = [&](const uint16_t* src, size_t base_par, uint32_t r, uint32_t c) -> uint32_t {
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
        return v;
    };
    // The words of tile t+1 are loaded into registers while tile t is written out.
    auto fetch = [&](uint32_t t, uint32_t (&w)[2 * kPairsPerThread]) {
        uint64_t b;
        uint32_t r0, c0;
        map.at(t, kT16, kT16, b, r0, c0);
        const uint16_t* src = in + b * map.mat;
        const size_t base_par = (b * map.mat) & 1;
#pragma unroll
        for (int k = 0; k < kPairsPerThread; ++k) {
            const uint32_t r = r0 + 2 * (ly + k * kRowsPerPass), c = c0 + 2 * lx;
            w[2 * k] = load_word(src, base_par, r, c);
            w[2 * k + 1] = load_word(src, base_par, r + 1, c);
        }
    };
    uint32_t w[2 * kPairsPerThread];
    uint32_t t = blockIdx.x;
    if (t < map.total) fetch(t, w);
    for (; t < map.total; t += gridDim.x) {
#pragma unroll
        for (int k = 0; k < kPairsPerThread; ++k) {
            const int p = ly + k * kRowsPerPass;
            blk[0][lx][p] = __byte_perm(w[2 * k], w[2 * k + 1], 0x5410);  // low halves: column c
            blk[1][lx][p] = __byte_perm(w[2 * k], w[2 * k + 1], 0x7632);  // high halves: column c + 1
        }
        __syncthreads();
        if (t + gridDim.x < map.total) fetch(t + gridDim.x, w);
        uint64_t b;
        uint32_t r0, c0;
        map.at(t, kT16, kT16, b, r0, c0);
        uint16_t* dst = out + b * map.mat;
        const size_t base_par = (b * map.mat) & 1;
        const uint32_t r = r0 + 2 * lx;
#pragma unroll
        for (int q = 0; q < kOutPerThread; ++q) {
            const int idx = ly + q * kRowsPerPass;  // 0..63: column pair idx >> 1, half idx & 1
            const int h = idx & 1, cp = idx >> 1;
            const uint32_t c = c0 + 2 * cp + h;
            if (c >= C) continue;
            const uint32_t v = blk[h][cp][lx];
            const size_t o = static_cast<size_t>(c) * R + r;
            if (r + 1 < R && ((base_par + o) & 1) == 0) {
                __stcs(reinterpret_cast<unsigned int*>(dst + o), v);
            } else {
                if (r < R) dst[o] = static_cast<uint16_t>(v);
                if (r + 1 < R) dst[o + 1] = static_cast<uint16_t>(v >> 16);
            }
        }
        __syncthreads();
    }
}

template <typename E>
int launch_transpose(const void* src, void* dst, uint32_t batch, uint32_t R, uint32_t C, void* stream) {
    TileMap map;
    if (!make_tile_map(map, batch, R, C, kTile, kTile))
        return fail(HC_ERR_INVALID, "transpose_2d_4d: %u matrices of %u x %u exceed 2^32 tiles", batch, R, C);
    const uint64_t cap = static_cast<uint64_t>(
        resident_blocks(reinterpret_cast<const void*>(transpose_kernel<E>), kTile * kRowsPerPass, 0));
    const int blocks = static_cast<int>(map.total < cap ? map.total : cap);
    if (blocks == 0) return ok();
    transpose_kernel<E><<<blocks, dim3(kTile, kRowsPerPass), 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const E*>(src), static_cast<E*>(dst), R, C, map);
    return check_launch("transpose_2d_4d");
}

// 2-byte elements with R and C multiples of 8 and 16-byte aligned buffers: tiles of 256 rows x 64
// columns arrive by TMA (128-byte swizzle) in a 3-stage ring, so up to three 32 KB tiles per block
// are in flight while one is written out.  Warp w owns tile rows 64 (w >> 1) .. +63 and 16-byte
// column chunks 4 (w & 1) .. +3.  Its lane (rb, jj) reads chunk j = 4 (w & 1) + jj of the eight rows
// row0 + i, row0 = 64 (w >> 1) + 8 rb (the 128-byte swizzle puts it in slot j ^ i), transposes that
// 8 x 8 block in registers (one byte permute per output word) and writes eight 16-byte words:
// output rows c0 + 8j + m, columns r0 + row0 .. +7.  The eight lanes with the same jj write one
// whole 128-byte line of an output row; a read costs eight wavefronts (four distinct slots per
// row), which shared memory absorbs easily at this traffic.
using namespace sm100;

constexpr uint32_t kTmaRows = 256, kTmaCols = 64, kTmaStages = 3, kTmaThreads = 256;
constexpr uint32_t kTmaTileBytes = kTmaRows * kTmaCols * 2;
constexpr size_t kTmaSmemBytes = kTmaStages * kTmaTileBytes + 1024;  // + alignment slack
constexpr uint32_t kErrTransposeWait = 1u, kErrTransposeDrain = 2u;
static_assert(kTmaRows == 64 * (kTmaThreads / 32 / 2) && kTmaCols == 64, "warp pairs cover 64 rows x 64 columns");

__device__ uint32_t g_transpose_error_word;

__global__ void __launch_bounds__(kTmaThreads) transpose16_tma_kernel(const __grid_constant__ CUtensorMap tm_in,
                                                                      uint16_t* __restrict__ out, uint32_t R,
                                                                      uint32_t C, TileMap map) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t full[kTmaStages];
    __shared__ uint32_t abort_flag;
    const uint32_t tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    if (tid == 0) {
        abort_flag = 0;
        for (uint32_t s = 0; s < kTmaStages; ++s) mbar_init(&full[s], 1);
        fence_mbar_init();
        prefetch_tmap(&tm_in);
    }
    __syncthreads();
    auto issue = [&](uint32_t t, uint32_t s) {
        uint64_t b;
        uint32_t r0, c0;
        map.at(t, kTmaRows, kTmaCols, b, r0, c0);
        mbar_arrive_expect_tx(&full[s], kTmaTileBytes);  // a box counts in full, zero-filled edges included
        tma_load_3d(smem + s * kTmaTileBytes, &tm_in, &full[s], static_cast<int32_t>(c0), static_cast<int32_t>(r0),
                    static_cast<int32_t>(b));
    };
    const uint64_t grid = gridDim.x;
    uint32_t issued = 0;  // tiles issued by thread 0 (only thread 0's count is used)
    if (tid == 0)
        for (uint32_t s = 0; s < kTmaStages && blockIdx.x + s * grid < map.total; ++s, ++issued)
            issue(static_cast<uint32_t>(blockIdx.x + s * grid), s);
    // warp w: tile rows 64 (w >> 1) .. +63, column chunks 4 (w & 1) .. +3; lane (rb, jj): 8 x 4
    const uint32_t rb = lane >> 2, j = 4 * (warp & 1) + (lane & 3);
    const uint32_t row0 = 64 * (warp >> 1) + rb * 8;  // first of this lane's eight tile rows (a multiple of 8)
    // Lanes of odd rb read their eight rows in the order 4..7, 0..3: a 16-byte shared-memory load is
    // served eight lanes at a time, and with the 128-byte swizzle the two rb of those eight lanes
    // then address disjoint bank quarters instead of the same ones (+2 % on B200).
    const uint32_t stag = 4 * (rb & 1);
    uint32_t k = 0;
    for (uint64_t t = blockIdx.x; t < map.total; t += grid, ++k) {
        const uint32_t s = k % kTmaStages;
        const bool ok = mbar_wait_bounded(&full[s], (k / kTmaStages) & 1u, &abort_flag, &g_transpose_error_word,
                                          kErrTransposeWait);
        if (ok) {
            uint64_t b;
            uint32_t r0, c0;
            map.at(static_cast<uint32_t>(t), kTmaRows, kTmaCols, b, r0, c0);
            const uint8_t* st = smem + s * kTmaTileBytes;
            uint32_t a[8][4];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                // a[i] holds tile row row0 + (i ^ stag), whose (row & 7) is i ^ stag: its chunk j sits
                // in slot j ^ (i ^ stag)
                const uint32_t ii = i ^ stag;
                const uint4 v = *reinterpret_cast<const uint4*>(st + (row0 + ii) * 128 + ((j ^ ii) << 4));
                a[i][0] = v.x;
                a[i][1] = v.y;
                a[i][2] = v.z;
                a[i][3] = v.w;
            }
            const uint32_t r = r0 + row0;
            if (r < R) {  // R % 8 == 0: the lane's eight rows are all inside or all outside
                uint16_t* dst = out + b * map.mat + r;
#pragma unroll
                for (int m = 0; m < 8; ++m) {
                    const uint32_t c = c0 + 8 * j + m;
                    if (c >= C) continue;
                    const uint32_t sel = (m & 1) ? 0x7632u : 0x5410u;  // high or low halves
                    const int w = m >> 1;
                    uint4 o;
                    o.x = __byte_perm(a[0][w], a[1][w], sel);
                    o.y = __byte_perm(a[2][w], a[3][w], sel);
                    o.z = __byte_perm(a[4][w], a[5][w], sel);
                    o.w = __byte_perm(a[6][w], a[7][w], sel);
                    if (stag) o = make_uint4(o.z, o.w, o.x, o.y);  // rows 4..7 came first
                    __stcs(reinterpret_cast<uint4*>(dst + static_cast<size_t>(c) * R), o);
                }
            }
        }
        // Every thread is done with stage s (or one of them gave up: then all leave together).
        if (!__syncthreads_and(ok)) break;
        if (tid == 0) {
            const uint64_t tn = t + kTmaStages * grid;
            if (tn < map.total) {
                issue(static_cast<uint32_t>(tn), s);
                ++issued;
            }
        }
    }
    // After a timeout, wait (bounded) for the copies still in flight before the block's shared
    // memory is released.
    if (tid == 0) {
        volatile uint32_t never = 0;
        for (uint32_t q = k; q < issued; ++q)
            mbar_wait_bounded(&full[q % kTmaStages], (q / kTmaStages) & 1u, &never, &g_transpose_error_word,
                              kErrTransposeDrain, 1000000000ull);
    }
}

uint32_t read_transpose_error_word(const char** name) {
    *name = "transpose_2d_4d";
    uint32_t word = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&word, g_transpose_error_word, sizeof(word)) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (word) cudaMemcpyToSymbol(g_transpose_error_word, &zero, sizeof(zero));
    return word;
}

// Returns false when the TMA path does not apply (the caller then takes transpose16_kernel);
// otherwise launches it and sets *status.
bool launch_transpose16_tma(const void* src, void* dst, uint32_t batch, uint32_t R, uint32_t C, void* stream,
                            int* status) {
    if ((reinterpret_cast<uintptr_t>(src) & 15) || (reinterpret_cast<uintptr_t>(dst) & 15) || (R & 7) || (C & 7))
        return false;
    TileMap map;
    if (!make_tile_map(map, batch, R, C, kTmaRows, kTmaCols)) return false;
    static std::once_flag once;
    std::call_once(once, [] { register_error_word(read_transpose_error_word); });
    *status = set_max_dynamic_smem(reinterpret_cast<const void*>(transpose16_tma_kernel), kTmaSmemBytes,
                                   "transpose16_tma_kernel");
    if (*status != HC_OK) return true;
    CUtensorMap tm;
    const uint64_t dims[3] = {C, R, batch};
    const uint64_t strides[2] = {static_cast<uint64_t>(C) * 2, static_cast<uint64_t>(R) * C * 2};
    const uint32_t box[3] = {kTmaCols, kTmaRows, 1};
    *status = encode_tmap(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, src, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (*status != HC_OK) return true;
    const uint64_t cap = static_cast<uint64_t>(
        resident_blocks(reinterpret_cast<const void*>(transpose16_tma_kernel), kTmaThreads, kTmaSmemBytes));
    const int blocks = static_cast<int>(map.total < cap ? map.total : cap);
    if (blocks == 0) {
        *status = ok();
        return true;
    }
    transpose16_tma_kernel<<<blocks, kTmaThreads, kTmaSmemBytes, static_cast<cudaStream_t>(stream)>>>(
        tm, static_cast<uint16_t*>(dst), R, C, map);
    *status = check_launch("transpose_2d_4d(tma)");
    return true;
}

int launch_transpose16(const void* src, void* dst, uint32_t batch, uint32_t R, uint32_t C, void* stream) {
    int status = HC_OK;
    if (launch_transpose16_tma(src, dst, batch, R, C, stream, &status)) return status;
    TileMap map;
    if (!make_tile_map(map, batch, R, C, kT16, kT16)) return launch_transpose<uint16_t>(src, dst, batch, R, C, stream);
    const uint64_t cap = static_cast<uint64_t>(
        resident_blocks(reinterpret_cast<const void*>(transpose16_kernel), kTile * kRowsPerPass, 0));
    const int blocks = static_cast<int>(map.total < cap ? map.total : cap);
    if (blocks == 0) return ok();
    transpose16_kernel<<<blocks, dim3(kTile, kRowsPerPass), 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t*>(src), static_cast<uint16_t*>(dst), R, C, map);
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
