// B200 drop-in for ops/flash_attention_fwd_fused/runner/flash_attention_fwd_fused_runner.hpp:1-21:
// the same entry point, executed on the GPU
// (harness::flash_attention_fwd_fused::run_flash_attention_fwd_fused_cuda; fp32 host buffers take
// the SIMT kernel, 16-bit device buffers the tcgen05 one through run_..._device).  The name keeps
// the reference's `_cpu` suffix so that the reference's tests and benches compile unchanged.
#pragma once
#include <cstdint>

#include "flash_attention_fwd_fused_golden.hpp"
#include "harness/device_ops.hpp"

namespace harness {
namespace flash_attention_fwd_fused {

inline void run_flash_attention_fwd_fused_cpu(const float* Q, const float* K, const float* V, float* O, int64_t B,
                                              int64_t H, int64_t S_q, int64_t S_k, int64_t D, int64_t D_v,
                                              float scale, AttnMaskType mask_type) {
    run_flash_attention_fwd_fused_cuda(Q, K, V, O, B, H, S_q, S_k, D, D_v, scale, static_cast<int>(mask_type));
}

}  // namespace flash_attention_fwd_fused
}  // namespace harness
