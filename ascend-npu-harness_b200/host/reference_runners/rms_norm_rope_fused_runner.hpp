// B200 drop-in for ops/rms_norm_rope_fused/runner/rms_norm_rope_fused_runner.hpp:1-22: the same
// entry point, executed on the GPU by the row-stream RMSNorm+RoPE kernel with the golden's
// interleaved pairing (harness::rms_norm_rope_fused::run_rms_norm_rope_fused_cuda).  The name keeps
// the reference's `_cpu` suffix so that the reference's tests and benches compile unchanged.
#pragma once
#include <cstdint>

#include "harness/device_ops.hpp"
#include "rms_norm_rope_fused_golden.hpp"

namespace harness {
namespace rms_norm_rope_fused {

inline void run_rms_norm_rope_fused_cpu(const float* x, const float* weight, const float* cos, const float* sin,
                                        float* out, int64_t B, int64_t S, int64_t H, int64_t rotary_dim, float eps) {
    run_rms_norm_rope_fused_cuda(x, weight, cos, sin, out, B, S, H, rotary_dim, eps);
}

}  // namespace rms_norm_rope_fused
}  // namespace harness
