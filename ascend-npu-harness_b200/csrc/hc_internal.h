// Internal helpers shared by the runtime shim and the operator launch files.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstddef>
#include <cstdint>

#include "hc_ops.h"
#include "hc_runtime.h"

namespace hc {

// Records `status` with a printf-style message as the calling thread's last error and
// returns the status, so call sites can `return fail(HC_ERR_INVALID, "...")`.
int fail(int status, const char* fmt, ...);

// Clears the thread's last error and returns HC_OK.
int ok();

// Converts a CUDA error into HC_ERR_CUDA with the call site in the message.
int cuda_fail(cudaError_t err, const char* what);

// Host-side fault injection (HC_FAULT="<call>:<n>").  Returns true when this call of
// `kind` ("malloc", "memcpy", "launch") must fail.
bool fault_hit(const char* kind);

// SM count of the current device (cached per device).
int sm_count();

// Blocks of `kernel` (launched with `threads` threads and `smem` bytes of dynamic shared memory)
// that are resident on the whole current device at once, from the occupancy calculator (cached
// per kernel, launch shape and device).  Grid-stride kernels use it as their grid cap: a larger
// grid leaves its extra blocks a second, partly empty wave at the end of the launch.
int resident_blocks(const void* kernel, int threads, size_t smem);

// Raises `kernel`'s dynamic shared-memory limit to at least `bytes` on the current device.
// cudaFuncSetAttribute acts on the current device's context only, so the setting is recorded per
// (kernel, device) under a lock: each device gets it on its first launch from any host thread,
// and threads driving different devices never share a flag.  Returns HC_OK or HC_ERR_CUDA
// naming `name`.
int set_max_dynamic_smem(const void* kernel, size_t bytes, const char* name);

// Checks a flash-attention tiling record, K/V head count and element type without touching the
// device (the checks hc_flash_attention_fwd_fused_gqa_launch makes before any launch).  An empty
// problem (B, H or S_q zero) is valid.  Returns HC_OK or the error status with its message set.
int fa_check_tiling(const flash_attention_fwd_fused_tiling_data* t, uint32_t kv_heads, int dtype);

// Unique id of the calling thread's current CUDA context (stable for the context's lifetime and
// never reused, unlike a device ordinal: a device reset gives the device a new id); 0 if unknown.
uint64_t current_context_id();

// Size in bytes of one element of an hc_dtype, 0 for an unknown value.
size_t dtype_size(int dtype);

// Checks a kernel launch: returns HC_OK or HC_ERR_CUDA naming `kernel`.
int check_launch(const char* kernel);

// Device error words: files whose kernels contain bounded spin-waits register a reader that
// copies and clears their word.  A non-zero word is reported by hc_check_device_error().
typedef uint32_t (*error_word_reader)(const char** kernel_name);
void register_error_word(error_word_reader reader);

}  // namespace hc

#define HC_CHECK_CUDA(call)                                          \
    do {                                                             \
        cudaError_t hc_err__ = (call);                               \
        if (hc_err__ != cudaSuccess) return hc::cuda_fail(hc_err__, #call); \
    } while (0)
