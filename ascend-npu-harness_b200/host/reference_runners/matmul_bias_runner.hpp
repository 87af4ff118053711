// B200 drop-in for ops/matmul_bias/runner/matmul_bias_runner.hpp:1-19: the same entry point,
// executed on the GPU (harness::matmul_bias::run_matmul_bias_cuda; fp32 host buffers take the SIMT
// GEMM).  The name keeps the reference's `_cpu` suffix so that the reference's tests and benches
// compile unchanged.
#pragma once
#include <cstdint>

#include "harness/device_ops.hpp"
#include "matmul_bias_golden.hpp"

namespace harness {
namespace matmul_bias {

inline void run_matmul_bias_cpu(const float* A, const float* B, const float* bias, float* C, int64_t M, int64_t K,
                                int64_t N) {
    run_matmul_bias_cuda(A, B, bias, C, M, K, N);
}

}  // namespace matmul_bias
}  // namespace harness
