// B200 definitions of the reference's elementwise-family runners and of its device-availability
// query, compiled against the reference's own headers.  Replaces, when linked with
// libhc_harness.so and libhc_b200.so:
//   ops/elementwise_add/runner/elementwise_add_runner.cpp:13-42
//   ops/axpy_scalar_affine/runner/axpy_scalar_affine_runner.cpp
//   ops/activation_gelu_silu/runner/activation_gelu_silu_runner.cpp
//   ops/reduce_sum_lastdim/runner/reduce_sum_lastdim_runner.cpp and
//   ops/broadcast_binary/runner/broadcast_binary_runner.cpp (their signatures already match
//   libhc_harness.so's definitions, so nothing is defined here for them)
//   harness::IsAscendRuntimeAvailable() of src/ascend_runtime.cpp (declared in
//   include/harness/skip.hpp:20-27; HasUsableDevice and GetDeviceCount come from
//   libhc_harness.so's device runtime)
// Each call runs on the GPU (copy in, kernel, copy out) and throws harness::DeviceError on
// failure; nothing falls back to the golden.
#include "activation_gelu_silu_runner.hpp"
#include "axpy_scalar_affine_runner.hpp"
#include "elementwise_add_runner.hpp"
#include "harness/device_ops.hpp"
#include "harness/shape.hpp"
#include "harness/skip.hpp"
#include "hc_runtime.h"

namespace harness {

bool IsAscendRuntimeAvailable() {
    int count = 0;
    return hc_init() == HC_OK && hc_device_count(&count) == HC_OK && count > 0;
}

namespace runner {

namespace elementwise_add {
void run(const float* x, const float* y, float* z, const Shape& shape) {
    run(x, y, z, static_cast<size_t>(shape.num_elements()));
}
}  // namespace elementwise_add

namespace axpy_scalar_affine {
void run(const float* x, float* y, const Shape& shape, float alpha, float beta) {
    run(x, y, static_cast<size_t>(shape.num_elements()), alpha, beta);
}
}  // namespace axpy_scalar_affine

namespace activation_gelu_silu {
void run(const float* x, float* y, const Shape& shape, golden::activation_gelu_silu::ActivationType act) {
    run(x, y, static_cast<size_t>(shape.num_elements()), static_cast<int>(act));
}
}  // namespace activation_gelu_silu

}  // namespace runner
}  // namespace harness
