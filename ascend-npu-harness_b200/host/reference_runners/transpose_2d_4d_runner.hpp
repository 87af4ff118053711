// B200 drop-in for ops/transpose_2d_4d/runner/transpose_2d_4d_runner.hpp:1-30: the same three
// entry points, executed on the GPU by the tiled transpose kernels
// (harness::transpose_2d_4d::run_transpose_*_cuda; any 1-, 2- or 4-byte element type, bit-exact).
// The names keep the reference's `_cpu` suffix so that the reference's tests and benches compile
// unchanged.
#pragma once
#include <cstdint>
#include <cstring>

#include "harness/device_ops.hpp"
#include "transpose_2d_4d_golden.hpp"
#include "transpose_2d_4d_tiling.hpp"

namespace harness {
namespace transpose_2d_4d {

template <typename T>
void run_transpose_2d_cpu(const T* input, T* output, int64_t M, int64_t N) {
    run_transpose_2d_cuda(input, output, M, N);
}

template <typename T>
void run_transpose_4d_nchw_to_nhwc_cpu(const T* input, T* output, int64_t N, int64_t C, int64_t H, int64_t W) {
    run_transpose_4d_nchw_to_nhwc_cuda(input, output, N, C, H, W);
}

template <typename T>
void run_transpose_4d_nhwc_to_nchw_cpu(const T* input, T* output, int64_t N, int64_t C, int64_t H, int64_t W) {
    run_transpose_4d_nhwc_to_nchw_cuda(input, output, N, C, H, W);
}

}  // namespace transpose_2d_4d
}  // namespace harness
