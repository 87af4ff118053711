// CPU tests of the C++ host layer: the accuracy pass rule, argument validation of the runners
// (done on the host before any device work), and the error behaviour without a device -- a
// DeviceError instead of the reference runners' silent fallback to the golden
// (ops/elementwise_add/runner/elementwise_add_runner.cpp:40-41).  Runs on machines with or
// without a GPU; the no-device expectations are skipped when a device is present.
#include <algorithm>
#include <string>
#include <vector>

#include "accuracy.hpp"
#include "harness/device_ops.hpp"
#include "harness/device_runtime.hpp"
#include "hc_ops.h"
#include "mini_gtest.hpp"

using harness::DeviceError;
using harness::accuracy::CompareArrays;
using harness::accuracy::Tolerance;

namespace {

template <class F>
int status_of(F&& f) {
    try {
        f();
    } catch (const DeviceError& e) {
        return e.status();
    }
    return HC_OK;
}

bool have_device() { return harness::device::GetDeviceCount() > 0; }

// Minimal shape object with the reference harness::Shape's num_elements().
struct TestShape {
    int64_t a, b;
    int64_t num_elements() const { return a * b; }
};

enum class TestActivation { GELU = 0, SiLU = 1 };
enum class TestMask { None = 0, Causal = 1 };

}  // namespace

// ================================================================ accuracy rule
TEST(AccuracyTest, FailsOnlyWhenAbsAndRelBothExceed) {
    std::vector<float> expected = {1000.0f, 1e-3f, 0.0f, 5.0f};
    std::vector<float> actual = {1000.5f, 1.5e-3f, 0.0f, 5.0f};
    // element 0: abs 0.5 > 1e-3 but rel 5e-4 <= 1e-3 -> passes; element 1: rel 0.5 but abs 5e-4 -> passes
    auto r = CompareArrays(expected, actual, Tolerance{1e-3, 1e-3});
    EXPECT_TRUE(r.passed) << r.ToString();
    EXPECT_NEAR(r.global_max_abs, 0.5, 1e-9);
    EXPECT_NEAR(r.global_max_rel, 0.5, 1e-6);
    actual[3] = 5.1f;
    auto r2 = CompareArrays(expected, actual, Tolerance{1e-3, 1e-3});
    EXPECT_FALSE(r2.passed);
    EXPECT_EQ(r2.mismatch_count, 1u);
    EXPECT_EQ(r2.first_mismatch, 3u);
}

TEST(AccuracyTest, ExactToleranceAndSizeMismatch) {
    std::vector<int> a = {1, 2, 3}, b = {1, 2, 3}, c = {1, 2};
    EXPECT_TRUE(CompareArrays(a, b, Tolerance{0, 0}).passed);
    EXPECT_FALSE(CompareArrays(a, c, Tolerance{0, 0}).passed);
    std::vector<float> x = {1.0f}, y = {std::nextafter(1.0f, 2.0f)};
    EXPECT_FALSE(CompareArrays(x, y, Tolerance{0, 0}).passed);
}

// ================================================================ runtime without device
TEST(HostRuntimeTest, ErrorNamesAndAlias) {
    EXPECT_EQ(std::string(harness::device::GetErrorString(HC_OK)), "HC_OK");
    EXPECT_EQ(std::string(harness::device::GetErrorString(HC_ERR_TIMEOUT)), "HC_ERR_TIMEOUT");
    EXPECT_EQ(std::string(harness::ascend::GetErrorString(HC_ERR_NO_DEVICE)), "HC_ERR_NO_DEVICE");
    EXPECT_EQ(harness::IsAscendRuntimeAvailable(), harness::IsDeviceRuntimeAvailable());
    EXPECT_EQ(harness::GetDeviceCount(), harness::device::GetDeviceCount());
}

TEST(HostRuntimeTest, NoDeviceReportsFailureWithoutThrowing) {
    if (have_device()) GTEST_SKIP() << "a CUDA device is present";
    EXPECT_FALSE(harness::device::RuntimeInit());
    EXPECT_FALSE(harness::device::IsAvailable());
    EXPECT_FALSE(harness::HasUsableDevice());
    EXPECT_EQ(harness::device::GetDeviceCount(), 0);
    EXPECT_TRUE(harness::device::DeviceMalloc(1024) == nullptr);
    EXPECT_TRUE(harness::device::CreateStream() == nullptr);
    EXPECT_TRUE(harness::device::CreateEvent() == nullptr);
    EXPECT_THROW(harness::device::DeviceMemory m(1024), std::runtime_error);
    harness::device::DeviceMemory empty(0);  // a zero-size buffer is not an error (reference semantics)
    EXPECT_FALSE(static_cast<bool>(empty));
}

TEST(HostRuntimeTest, RunnersThrowInsteadOfFallingBack) {
    if (have_device()) GTEST_SKIP() << "a CUDA device is present";
    std::vector<float> x = {1.0f, 2.0f}, y = {3.0f, 4.0f}, z = {-7.0f, -7.0f};
    EXPECT_EQ(status_of([&] { harness::runner::elementwise_add::run(x.data(), y.data(), z.data(), 2); }),
              HC_ERR_NO_DEVICE);
    EXPECT_EQ(status_of([&] { harness::runner::elementwise_add::run(x.data(), y.data(), z.data(), TestShape{1, 2}); }),
              HC_ERR_NO_DEVICE);
    EXPECT_EQ(status_of([&] { harness::runner::activation_gelu_silu::run(x.data(), z.data(), 2, TestActivation::SiLU); }),
              HC_ERR_NO_DEVICE);
    EXPECT_EQ(status_of([&] { harness::layer_norm::run_layer_norm_cuda(x.data(), x.data(), y.data(), z.data(), 1, 2, 1e-5f); }),
              HC_ERR_NO_DEVICE);
    EXPECT_EQ(status_of([&] {
                  harness::flash_attention_fwd_fused::run_flash_attention_fwd_fused_cuda(
                      x.data(), x.data(), y.data(), z.data(), 1, 1, 1, 1, 2, 2, 0.5f, TestMask::Causal);
              }),
              HC_ERR_NO_DEVICE);
    EXPECT_TRUE(z[0] == -7.0f && z[1] == -7.0f) << "nothing may be computed on the CPU";
}

// ================================================================ host-side validation
TEST(HostValidationTest, ArgumentsTheKernelsCannotTakeAreRejectedFirst) {
    std::vector<float> b(16, 0.0f);
    EXPECT_EQ(status_of([&] { harness::runner::activation_gelu_silu::run(b.data(), b.data(), 4, 2); }), HC_ERR_INVALID);
    EXPECT_EQ(status_of([&] { harness::runner::broadcast_binary::run(b.data(), b.data(), b.data(), b.data(), 2, 2, 2, 2, 3); }),
              HC_ERR_INVALID);
    EXPECT_EQ(status_of([&] {
                  harness::rms_norm_rope_fused::run_rms_norm_rope_fused_cuda(b.data(), b.data(), b.data(), b.data(),
                                                                             b.data(), 1, 1, 8, 5, 1e-6f);
              }),
              HC_ERR_INVALID);
    EXPECT_EQ(status_of([&] {
                  harness::flash_attention_fwd_fused::run_flash_attention_fwd_fused_cuda(
                      b.data(), b.data(), b.data(), b.data(), 1, 1, 1, 1, 2, 2, 0.5f, 2);
              }),
              HC_ERR_INVALID);
    EXPECT_EQ(status_of([&] {
                  harness::flash_attention_fwd_fused::run_flash_attention_fwd_fused_gqa_device(
                      b.data(), b.data(), b.data(), b.data(), nullptr, 1, 8, 3, 16, 16, 128, 128, 0.5f, 1,
                      harness::device::Dtype::BF16);
              }),
              HC_ERR_INVALID)
        << "kv_heads must divide H (checked before any device work)";
    EXPECT_EQ(status_of([&] { harness::runner::reduce_sum_lastdim::run(b.data(), b.data(), 1, -1, 4); }), HC_ERR_INVALID);
    EXPECT_EQ(status_of([&] {
                  harness::matmul_bias::run_matmul_bias_cuda(b.data(), b.data(), nullptr, b.data(), int64_t(1) << 20,
                                                             int64_t(1) << 13, 1);
              }),
              HC_ERR_INVALID)
        << "M*K beyond the 32-bit tiling field";
    EXPECT_EQ(status_of([&] {
                  harness::transpose_2d_4d::run_transpose_host(b.data(), b.data(), 0, 2, 2, 1, 1, 8);
              }),
              HC_ERR_UNSUPPORTED);
}

TEST(HostValidationTest, EmptyInputsAreANoOp) {
    if (!have_device()) GTEST_SKIP() << "empty inputs still require a device (no CPU path)";
    std::vector<float> z = {-7.0f};
    EXPECT_NO_THROW(harness::runner::elementwise_add::run(z.data(), z.data(), z.data(), 0));
    EXPECT_FLOAT_EQ(z[0], -7.0f);
}

MINI_GTEST_MAIN
