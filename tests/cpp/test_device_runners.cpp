// GPU parity tests of the C++ host layer (harness::device runtime and the per-op runners in
// ascend-npu-harness_b200/host/include/harness/device_ops.hpp) against the CPU oracle.
//
// The cases, seeds, value ranges and tolerances are the reference harness's own
// (tests/test_<op>.cpp of z-zijie/ascend-npu-harness); the only change is that the runner under
// test executes the CUDA kernel instead of the golden.  fp32 host-pointer runners are checked on
// every reference case; the bf16 device-pointer and host-buffer calls are checked on the
// tensor-core shapes.  Needs a CUDA device (run through tests/test_gpu_cpp_runners.py).
#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "accuracy.hpp"
#include "harness/device_ops.hpp"
#include "harness/device_runtime.hpp"
#include "hc_ops.h"
#include "mini_gtest.hpp"
#include "oracle.h"
#include "test_util.hpp"

using harness::DeviceError;
using harness::accuracy::CompareArrays;
using harness::accuracy::Tolerance;
using harness::device::DeviceMemory;
using harness::device::Dtype;
using namespace hc_test;

namespace {

constexpr Tolerance kExact{0.0, 0.0};

// Uploads a host vector into a new device buffer.
template <class T>
DeviceMemory upload(const std::vector<T>& h) {
    DeviceMemory d(h.size() * sizeof(T));
    EXPECT_TRUE(harness::device::MemcpyHostToDevice(d.data(), h.data(), h.size() * sizeof(T)));
    return d;
}

template <class T>
std::vector<T> download(const DeviceMemory& d, size_t n) {
    std::vector<T> h(n);
    EXPECT_TRUE(harness::device::MemcpyDeviceToHost(h.data(), d.data(), n * sizeof(T)));
    return h;
}

float default_scale(int64_t D) { return 1.0f / std::sqrt(static_cast<float>(D)); }

}  // namespace

// ================================================================ runtime
TEST(DeviceRuntimeTest, InitCountAndMemory) {
    ASSERT_TRUE(harness::device::RuntimeInit());
    ASSERT_TRUE(harness::HasUsableDevice());
    ASSERT_GE(harness::device::GetDeviceCount(), 1);
    ASSERT_TRUE(harness::ascend::SetDevice(0));  // the reference's spelling resolves to the same layer
    EXPECT_EQ(harness::device::GetCurrentDevice(), 0);
    EXPECT_FALSE(harness::device::GetDriverVersion().empty());
    EXPECT_NE(harness::device::GetSocVersion().find("sm_"), std::string::npos) << harness::device::GetSocVersion();

    std::vector<float> h = uniform(4097, kSeed), back(4097, 0.0f);
    DeviceMemory d(h.size() * sizeof(float));
    ASSERT_TRUE(static_cast<bool>(d));
    EXPECT_TRUE(harness::device::MemcpyHostToDevice(d.data(), h.data(), h.size() * 4));
    EXPECT_TRUE(harness::device::MemcpyDeviceToHost(back.data(), d.data(), h.size() * 4));
    EXPECT_TRUE(h == back);
    DeviceMemory moved(std::move(d));
    EXPECT_FALSE(static_cast<bool>(d));
    EXPECT_EQ(moved.size(), h.size() * 4);
}

TEST(DeviceRuntimeTest, StreamsAndEventsTime) {
    auto stream = harness::device::CreateStream();
    ASSERT_TRUE(stream != nullptr);
    auto start = harness::device::CreateEvent(), stop = harness::device::CreateEvent();
    ASSERT_TRUE(start != nullptr && stop != nullptr);
    const size_t n = 1 << 24;
    std::vector<float> x = uniform(n, kSeed);
    DeviceMemory dx = upload(x), dy(n * 4);
    EXPECT_TRUE(harness::device::RecordEvent(start.get(), stream.get()));
    harness::runner::axpy_scalar_affine::run_device(dx.data(), dy.data(), n, 2.0f, 1.0f, Dtype::F32, stream.get());
    EXPECT_TRUE(harness::device::RecordEvent(stop.get(), stream.get()));
    EXPECT_TRUE(harness::device::EventSynchronize(stop.get()));
    float ms = -1.0f;
    EXPECT_TRUE(harness::device::EventElapsedTime(&ms, start.get(), stop.get()));
    EXPECT_GT(ms, 0.0f);
    EXPECT_TRUE(harness::device::StreamSynchronize(stream.get()));
    EXPECT_TRUE(harness::device::CheckDeviceError());
}

TEST(DeviceRuntimeTest, ExpiredBoundedWaitIsReported) {
    EXPECT_EQ(hc_selftest_bounded_wait(1000), HC_ERR_TIMEOUT);
    EXPECT_TRUE(harness::device::CheckDeviceError()) << "the error word is read and cleared by the self-test";
    // the context stays usable: a kernel still runs afterwards
    std::vector<float> x = {1.0f, 2.0f}, y = {3.0f, 4.0f}, z(2);
    harness::runner::elementwise_add::run(x.data(), y.data(), z.data(), 2);
    EXPECT_FLOAT_EQ(z[1], 6.0f);
}

TEST(DeviceRuntimeTest, InjectedFailureThrowsAndNothingFallsBack) {
    std::vector<float> x = uniform(64, kSeed), y = uniform(64, kSeed + 1), z(64, -7.0f);
    ASSERT_EQ(hc_set_fault("malloc:2"), HC_OK);
    int status = HC_OK;
    try {
        harness::runner::elementwise_add::run(x.data(), y.data(), z.data(), z.size());
    } catch (const DeviceError& e) {
        status = e.status();
    }
    hc_set_fault(nullptr);
    EXPECT_EQ(status, HC_ERR_INJECTED);
    EXPECT_TRUE(std::all_of(z.begin(), z.end(), [](float v) { return v == -7.0f; })) << "output must stay untouched";
}

// ================================================================ elementwise_add
TEST(ElementwiseAddTest, SimpleValues) {  // tests/test_elementwise_add.cpp:19-28
    std::vector<float> x = {1.0f, 2.0f, 3.0f, 4.0f}, y = {5.0f, 6.0f, 7.0f, 8.0f}, z(4);
    harness::runner::elementwise_add::run(x.data(), y.data(), z.data(), 4);
    std::vector<float> expected = {6.0f, 8.0f, 10.0f, 12.0f};
    EXPECT_TRUE(CompareArrays(expected, z, kExact).passed);
}

TEST(ElementwiseAddTest, ReferenceShapesBitExact) {  // tests/test_elementwise_add.cpp:81-89
    const std::vector<std::vector<int64_t>> shapes = {{1}, {8}, {1024}, {3, 7}, {4, 16, 64}, {2, 3, 32, 128}};
    for (const auto& s : shapes) {
        size_t n = 1;
        for (auto d : s) n *= d;
        auto x = uniform(n, kSeed), y = uniform(n, kSeed + 1);
        std::vector<float> z(n), ref(n);
        harness::runner::elementwise_add::run(x.data(), y.data(), z.data(), n);
        oracle_elementwise_add(x.data(), y.data(), ref.data(), n);
        auto r = CompareArrays(ref, z, kExact);
        EXPECT_TRUE(r.passed) << "n=" << n << " " << r.ToString();
    }
}

TEST(ElementwiseAddTest, Bf16DeviceBuffersBitExact) {
    const size_t n = 4096 * 33 + 5;
    auto xq = to_bf16(uniform(n, 0)), yq = to_bf16(uniform(n, 1));
    DeviceMemory dx = upload(xq), dy = upload(yq), dz(n * 2);
    harness::runner::elementwise_add::run_device(dx.data(), dy.data(), dz.data(), n, Dtype::BF16);
    ASSERT_TRUE(harness::device::DeviceSynchronize());
    auto got = download<uint16_t>(dz, n);
    std::vector<float> ref(n);
    auto xf = from_bf16(xq), yf = from_bf16(yq);
    oracle_elementwise_add(xf.data(), yf.data(), ref.data(), n);
    EXPECT_TRUE(got == to_bf16(ref));
}

// ================================================================ axpy_scalar_affine
TEST(AxpyScalarAffineTest, ReferenceCasesBitExact) {  // tests/test_axpy_scalar_affine.cpp:93-111
    const size_t sizes[] = {1, 17, 1024, 4097, 32 * 128};
    const float scalars[] = {0.0f, 1.0f, -1.0f, 0.5f, -2.25f};
    for (size_t n : sizes)
        for (float a : scalars)
            for (float b : scalars) {
                auto x = uniform(n, kSeed);
                std::vector<float> y(n), ref(n);
                harness::runner::axpy_scalar_affine::run(x.data(), y.data(), n, a, b);
                oracle_axpy_scalar_affine(x.data(), ref.data(), n, a, b);
                EXPECT_TRUE(CompareArrays(ref, y, kExact).passed) << "n=" << n << " alpha=" << a << " beta=" << b;
            }
}

// ================================================================ broadcast_binary
TEST(BroadcastBinaryTest, ReferenceCasesBitExact) {  // tests/test_broadcast_binary.cpp:116-128
    const int64_t cases[][5] = {{1, 1, 1, 1, 1},   {1, 3, 7, 7, 1},  {2, 16, 32, 32, 1}, {4, 64, 63, 63, 1},
                                {1, 3, 32, 64, 1}, {2, 1, 32, 32, 2}, {1, 1, 63, 63, 1},  {4, 16, 1, 1, 1},
                                {1, 64, 7, 7, 1}};
    for (const auto& c : cases) {
        const int64_t B = c[0], C = c[1], H = c[2], W = c[3], yb = c[4];
        const size_t n = prod({B, C, H, W});
        auto x = uniform(n, kSeed), y = uniform(yb * C, kSeed + 1), bias = uniform(C, kSeed + 2);
        std::vector<float> z(n), ref(n);
        harness::runner::broadcast_binary::run(x.data(), y.data(), bias.data(), z.data(), B, C, H, W, yb);
        oracle_broadcast_binary(x.data(), y.data(), bias.data(), ref.data(), B, C, H, W, yb);
        EXPECT_TRUE(CompareArrays(ref, z, kExact).passed) << B << "x" << C << "x" << H << "x" << W << " yb=" << yb;
    }
}

// ================================================================ activation_gelu_silu
TEST(ActivationGeluSiluTest, ReferenceCases) {  // tests/test_activation_gelu_silu.cpp:59-69
    const struct {
        size_t n;
        int act;
    } cases[] = {{128, 0}, {1024, 0}, {8 * 512, 1}, {2 * 16 * 128, 1}, {1 << 20, 0}, {1 << 20, 1}};
    for (const auto& c : cases) {
        auto x = uniform(c.n, kSeed, -8.0f, 8.0f);
        std::vector<float> y(c.n), ref(c.n);
        harness::runner::activation_gelu_silu::run(x.data(), y.data(), c.n, c.act);
        oracle_activation_gelu_silu(x.data(), ref.data(), c.n, c.act);
        auto r = CompareArrays(ref, y, Tolerance{1e-5, 1e-5});
        EXPECT_TRUE(r.passed) << "n=" << c.n << " act=" << c.act << " " << r.ToString();
    }
}

TEST(ActivationGeluSiluTest, SpecValues) {  // tests/test_activation_gelu_silu.cpp:28-44
    std::vector<float> x = {-20.0f, -10.0f, -5.0f, -1.0f, 0.0f, 1.0f, 5.0f, 10.0f, 20.0f};
    for (int act : {0, 1}) {
        std::vector<float> y(x.size()), ref(x.size());
        harness::runner::activation_gelu_silu::run(x.data(), y.data(), x.size(), act);
        oracle_activation_gelu_silu(x.data(), ref.data(), x.size(), act);
        EXPECT_TRUE(CompareArrays(ref, y, Tolerance{1e-5, 1e-5}).passed) << "act=" << act;
    }
}

// ================================================================ reduce_sum_lastdim
TEST(ReduceSumLastdimTest, ReferenceCases) {  // tests/test_reduce_sum_lastdim.cpp:114-165
    const int64_t cases[][3] = {{1, 1, 1},    {1, 1, 7},   {1, 1, 32},   {1, 1, 128},    {1, 1, 1024}, {1, 1, 4096},
                                {1, 3, 128},  {1, 64, 32}, {1, 64, 4096}, {1, 257, 7},   {2, 3, 128},  {8, 64, 1024},
                                {1, 64, 1},   {2, 1, 4096}, {8, 1, 7},   {1, 2, 100000}, {1, 16384, 4096}};
    for (const auto& c : cases) {
        const int64_t B = c[0], M = c[1], K = c[2];
        auto x = uniform(prod({B, M, K}), kSeed);
        std::vector<float> out(B * M), ref(B * M);
        harness::runner::reduce_sum_lastdim::run(x.data(), out.data(), B, M, K);
        oracle_reduce_sum_lastdim(x.data(), ref.data(), B, M, K);
        auto r = CompareArrays(ref, out, Tolerance{1e-4, 1e-4});
        EXPECT_TRUE(r.passed) << B << "x" << M << "x" << K << " " << r.ToString();
    }
}

TEST(ReduceSumLastdimTest, KnownAnswers) {  // tests/test_reduce_sum_lastdim.cpp:20-85, 175-187
    std::vector<float> x = {1, 2, 3, 4, 5, 6}, out(2);
    harness::runner::reduce_sum_lastdim::run(x.data(), out.data(), 1, 2, 3);
    EXPECT_FLOAT_EQ(out[0], 6.0f);
    EXPECT_FLOAT_EQ(out[1], 15.0f);
    std::vector<float> ones(100000, 1.0f), s(1);
    harness::runner::reduce_sum_lastdim::run(ones.data(), s.data(), 1, 1, 100000);
    EXPECT_NEAR(s[0], 100000.0f, 1.0f);
}

// ================================================================ transpose_2d_4d
TEST(Transpose2d4dTest, TwoDimensionalBitExact) {  // tests/test_transpose_2d_4d.cpp:48-75
    const int64_t cases[][2] = {{1, 1}, {3, 7}, {32, 32}, {128, 64}, {257, 129}, {4096, 4100}};
    for (const auto& c : cases) {
        const int64_t M = c[0], N = c[1];
        auto x = uniform(M * N, kSeed);
        std::vector<float> y(M * N), ref(M * N);
        harness::transpose_2d_4d::run_transpose_2d_cuda(x.data(), y.data(), M, N);
        oracle_transpose(x.data(), ref.data(), 0, M, N, 1, 1, 4);
        EXPECT_TRUE(CompareArrays(ref, y, kExact).passed) << M << "x" << N;
        std::vector<int32_t> xi(M * N), yi(M * N), refi(M * N);
        for (int64_t i = 0; i < M * N; ++i) xi[i] = static_cast<int32_t>(i * 7 - 3);
        harness::transpose_2d_4d::run_transpose_2d_cuda(xi.data(), yi.data(), M, N);
        oracle_transpose(xi.data(), refi.data(), 0, M, N, 1, 1, 4);
        EXPECT_TRUE(yi == refi) << "int32 " << M << "x" << N;
    }
}

TEST(Transpose2d4dTest, FourDimensionalRoundTrip) {  // tests/test_transpose_2d_4d.cpp:80-126
    const int64_t cases[][4] = {{1, 3, 224, 224}, {2, 16, 32, 32}, {4, 7, 13, 17}};
    for (const auto& c : cases) {
        const int64_t N = c[0], C = c[1], H = c[2], W = c[3];
        auto x = uniform(prod({N, C, H, W}), kSeed);
        std::vector<float> nhwc(x.size()), ref(x.size()), back(x.size());
        harness::transpose_2d_4d::run_transpose_4d_nchw_to_nhwc_cuda(x.data(), nhwc.data(), N, C, H, W);
        oracle_transpose(x.data(), ref.data(), 1, N, C, H, W, 4);
        EXPECT_TRUE(nhwc == ref) << N << "x" << C << "x" << H << "x" << W;
        harness::transpose_2d_4d::run_transpose_4d_nhwc_to_nchw_cuda(nhwc.data(), back.data(), N, C, H, W);
        EXPECT_TRUE(back == x) << "round trip";
    }
}

// ================================================================ layer_norm
TEST(LayerNormTest, ReferenceCases) {  // tests/test_layer_norm.cpp:27-56
    const struct {
        int64_t rows, dim;
        float eps;
    } cases[] = {{1, 16, 1e-5f},   {3, 64, 1e-5f},   {1, 128, 1e-5f},   {64, 768, 1e-5f}, {4, 1024, 1e-5f},
                 {1, 4096, 1e-5f}, {257, 64, 1e-5f}, {1, 64, 1e-5f},    {16, 768, 1e-5f}, {32, 256, 1e-5f},
                 {512, 128, 1e-5f}, {64, 768, 1e-6f}, {3, 100, 1e-5f}, {2, 40000, 1e-5f}};
    for (const auto& c : cases) {
        auto x = uniform(c.rows * c.dim, kSeed, -3.0f, 3.0f);
        auto g = uniform(c.dim, kSeed + 1, 0.5f, 1.5f), b = uniform(c.dim, kSeed + 2, -0.5f, 0.5f);
        std::vector<float> y(x.size()), ref(x.size());
        harness::layer_norm::run_layer_norm_cuda(x.data(), g.data(), b.data(), y.data(), c.rows, c.dim, c.eps);
        oracle_layer_norm(x.data(), g.data(), b.data(), ref.data(), c.rows, c.dim, c.eps);
        auto r = CompareArrays(ref, y, Tolerance{1e-4, 1e-4});
        EXPECT_TRUE(r.passed) << c.rows << "x" << c.dim << " " << r.ToString();
    }
}

TEST(LayerNormTest, ConstantRowGivesBeta) {  // tests/test_layer_norm.cpp:61-89
    std::vector<float> x(4 * 128, 3.5f), y(x.size());
    auto g = uniform(128, 99, 0.5f, 1.5f), b = uniform(128, 100, -0.5f, 0.5f);
    harness::layer_norm::run_layer_norm_cuda(x.data(), g.data(), b.data(), y.data(), 4, 128, 1e-5f);
    for (size_t i = 0; i < y.size(); ++i) EXPECT_NEAR(y[i], b[i % 128], 1e-4) << "at " << i;
}

// ================================================================ rms_norm_rope_fused
TEST(RmsNormRopeFusedTest, ReferenceCases) {  // tests/test_rms_norm_rope_fused.cpp:19-48
    const struct {
        int64_t B, S, H, rot;
        float eps;
    } cases[] = {{1, 1, 64, 32, 1e-5f},   {1, 16, 128, 64, 1e-5f}, {2, 16, 256, 128, 1e-5f},
                 {4, 128, 128, 64, 1e-5f}, {1, 16, 128, 64, 1e-6f}, {1, 16, 64, 64, 1e-5f}};
    for (const auto& c : cases) {
        auto x = uniform(prod({c.B, c.S, c.H}), kSeed), w = uniform(c.H, kSeed + 1);
        std::vector<float> cs(c.S * c.rot / 2), sn(cs.size());
        oracle_rope_cos_sin(c.S, c.rot / 2, cs.data(), sn.data(), 10000.0f);
        std::vector<float> out(x.size()), ref(x.size());
        harness::rms_norm_rope_fused::run_rms_norm_rope_fused_cuda(x.data(), w.data(), cs.data(), sn.data(), out.data(),
                                                                   c.B, c.S, c.H, c.rot, c.eps);
        oracle_rms_norm_rope(x.data(), w.data(), cs.data(), sn.data(), ref.data(), c.B * c.S, c.H, c.rot, c.eps, 1, c.S, 0);
        auto r = CompareArrays(ref, out, Tolerance{1e-4, 1e-4});
        EXPECT_TRUE(r.passed) << c.B << "x" << c.S << "x" << c.H << " rot " << c.rot << " " << r.ToString();
    }
}

TEST(RmsNormRopeFusedTest, Bf16RotateHalfHeadsOnDevice) {
    const int64_t B = 2, S = 257, Hh = 32, D = 128;
    const size_t n = prod({B, S, Hh, D});
    auto xq = to_bf16(normal(n, 0));
    auto w = uniform(D, 1, 0.5f, 1.5f);
    std::vector<float> cs(S * D / 2), sn(cs.size());
    oracle_rope_cos_sin(S, D / 2, cs.data(), sn.data(), 10000.0f);
    DeviceMemory dx = upload(xq), dw = upload(w), dc = upload(cs), ds = upload(sn), dy(n * 2);
    harness::rms_norm_rope_fused::run_rms_norm_rope_fused_device(
        dx.data(), dw.as<float>(), dc.as<float>(), ds.as<float>(), dy.data(), B, S, D, D, 1e-6f, Hh,
        harness::rms_norm_rope_fused::RopeStyle::RotateHalf, Dtype::BF16);
    ASSERT_TRUE(harness::device::DeviceSynchronize());
    auto got = from_bf16(download<uint16_t>(dy, n));
    auto xf = from_bf16(xq);
    std::vector<float> ref(n);
    oracle_rms_norm_rope(xf.data(), w.data(), cs.data(), sn.data(), ref.data(), B * S * Hh, D, D, 1e-6f, Hh, S, 1);
    auto r = CompareArrays(ref, got, Tolerance{2e-2, 1.0 / 256});  // max-abs 2e-2, or half a bf16 ulp
    EXPECT_TRUE(r.passed) << r.ToString();
}

// ================================================================ matmul_bias
TEST(MatmulBiasTest, ReferenceCases) {  // tests/test_matmul_bias.cpp:22-67
    const struct {
        int64_t M, K, N;
        bool bias;
    } cases[] = {{1, 1, 1, false},     {16, 16, 16, false},   {64, 64, 64, false},   {128, 128, 128, false},
                 {256, 64, 16, false}, {1, 1024, 64, false},  {1, 1, 1, true},       {16, 16, 16, true},
                 {64, 32, 128, true},  {128, 128, 128, true}, {256, 256, 64, true},  {1, 1024, 64, true},
                 {64, 64, 1, false},   {1, 1, 64, false},     {1, 1024, 1, true}};
    for (const auto& c : cases) {
        auto A = uniform(c.M * c.K, kSeed, -2.0f, 2.0f), Bm = uniform(c.K * c.N, kSeed + 1, -2.0f, 2.0f);
        auto bias = uniform(c.N, kSeed + 2, -0.5f, 0.5f);
        std::vector<float> C(c.M * c.N), ref(C.size());
        harness::matmul_bias::run_matmul_bias_cuda(A.data(), Bm.data(), c.bias ? bias.data() : nullptr, C.data(), c.M,
                                                   c.K, c.N);
        oracle_matmul_bias(A.data(), Bm.data(), c.bias ? bias.data() : nullptr, ref.data(), c.M, c.K, c.N);
        auto r = CompareArrays(ref, C, Tolerance{1e-4, 1e-4});
        EXPECT_TRUE(r.passed) << c.M << "x" << c.K << "x" << c.N << " " << r.ToString();
    }
}

TEST(MatmulBiasTest, Bf16TensorCoreOnDevice) {
    const int64_t M = 1000, K = 1024, N = 1000;
    auto Aq = to_bf16(uniform(M * K, kSeed, -2.0f, 2.0f)), Bq = to_bf16(uniform(K * N, kSeed + 1, -2.0f, 2.0f));
    auto bq = to_bf16(uniform(N, kSeed + 2, -0.5f, 0.5f));
    DeviceMemory dA = upload(Aq), dB = upload(Bq), db = upload(bq), dC(M * N * 2);
    harness::matmul_bias::run_matmul_bias_device(dA.data(), dB.data(), db.data(), dC.data(), M, K, N, Dtype::BF16);
    ASSERT_TRUE(harness::device::DeviceSynchronize());
    EXPECT_EQ(hc_matmul_bias_last_path(), 3) << "bf16 with K, N multiples of 8 and M >= 256 takes the tcgen05 CTA-pair kernel";
    auto got = from_bf16(download<uint16_t>(dC, M * N));
    auto Af = from_bf16(Aq), Bf = from_bf16(Bq), bf = from_bf16(bq);
    std::vector<float> ref(M * N);
    oracle_matmul_bias(Af.data(), Bf.data(), bf.data(), ref.data(), M, K, N);
    double max_ref = 0, max_err = 0;
    for (size_t i = 0; i < ref.size(); ++i) {
        max_ref = std::max(max_ref, std::fabs(static_cast<double>(ref[i])));
        max_err = std::max(max_err, std::fabs(static_cast<double>(ref[i]) - got[i]));
    }
    EXPECT_LE(max_err / max_ref, 1e-2) << "rel-err vs the fp32 golden";
}

// ================================================================ flash_attention_fwd_fused
TEST(FlashAttentionTest, ReferenceCasesF32) {  // tests/test_flash_attention_fwd_fused.cpp:69-178
    const int64_t cases[][7] = {{1, 4, 1, 1, 32, 32, 0},     {1, 1, 16, 16, 64, 64, 0},   {1, 8, 16, 16, 32, 32, 0},
                                {2, 4, 16, 16, 64, 64, 0},   {1, 4, 8, 8, 32, 32, 1},     {1, 1, 16, 16, 64, 64, 1},
                                {2, 4, 32, 32, 128, 128, 1}, {1, 4, 8, 16, 64, 64, 0},    {1, 2, 4, 32, 128, 128, 0},
                                {1, 4, 64, 64, 64, 64, 0},   {1, 4, 64, 64, 64, 64, 1},   {1, 2, 128, 128, 32, 32, 0},
                                {1, 4, 8, 8, 64, 32, 0},     {1, 4, 16, 16, 128, 64, 1}};
    for (const auto& c : cases) {
        const int64_t B = c[0], H = c[1], Sq = c[2], Sk = c[3], D = c[4], Dv = c[5];
        const int mask = static_cast<int>(c[6]);
        auto q = uniform(prod({B, H, Sq, D}), kSeed), k = uniform(prod({B, H, Sk, D}), kSeed + 1000),
             v = uniform(prod({B, H, Sk, Dv}), kSeed + 2000);
        std::vector<float> o(prod({B, H, Sq, Dv})), ref(o.size());
        const float sc = default_scale(D);
        harness::flash_attention_fwd_fused::run_flash_attention_fwd_fused_cuda(q.data(), k.data(), v.data(), o.data(),
                                                                               B, H, Sq, Sk, D, Dv, sc, mask);
        oracle_flash_attention_fwd(q.data(), k.data(), v.data(), ref.data(), nullptr, B, H, Sq, Sk, D, Dv, sc, mask);
        auto r = CompareArrays(ref, o, Tolerance{5e-4, 5e-4});
        EXPECT_TRUE(r.passed) << "B" << B << " H" << H << " Sq" << Sq << " Sk" << Sk << " D" << D << " Dv" << Dv
                              << " mask " << mask << " " << r.ToString();
    }
}

TEST(FlashAttentionTest, Bf16SubsliceOnTensorCores) {  // B=1 H=2 S=1024 D=128, N(0,1) seeds 0/1/2
    const int64_t B = 1, H = 2, S = 1024, D = 128;
    const size_t n = prod({B, H, S, D});
    auto qq = to_bf16(normal(n, 0)), kq = to_bf16(normal(n, 1)), vq = to_bf16(normal(n, 2));
    auto qf = from_bf16(qq), kf = from_bf16(kq), vf = from_bf16(vq);
    const float sc = default_scale(D);
    DeviceMemory dq = upload(qq), dk = upload(kq), dv = upload(vq), dout(n * 2), dlse(B * H * S * 4);
    for (int mask : {1, 0}) {
        harness::flash_attention_fwd_fused::run_flash_attention_fwd_fused_device(
            dq.data(), dk.data(), dv.data(), dout.data(), dlse.as<float>(), B, H, S, S, D, D, sc, mask, Dtype::BF16);
        ASSERT_TRUE(harness::device::DeviceSynchronize());
        ASSERT_TRUE(harness::device::CheckDeviceError());
        EXPECT_EQ(hc_flash_attention_last_path(), 1) << "D=128 bf16 takes the tcgen05/TMEM kernel";
        auto o = from_bf16(download<uint16_t>(dout, n));
        auto lse = download<float>(dlse, B * H * S);
        std::vector<float> ref(n), ref_lse(B * H * S);
        oracle_flash_attention_fwd(qf.data(), kf.data(), vf.data(), ref.data(), ref_lse.data(), B, H, S, S, D, D, sc,
                                   mask);
        auto r = CompareArrays(ref, o, Tolerance{2e-2, 0.0});
        EXPECT_TRUE(r.passed) << "mask " << mask << " " << r.ToString();
        auto rl = CompareArrays(ref_lse, lse, Tolerance{2e-3, 0.0});
        EXPECT_TRUE(rl.passed) << "lse mask " << mask << " " << rl.ToString();
    }
}

TEST(FlashAttentionTest, GroupedQueryMatchesRepeatedHeads) {
    // 8 query heads over 2 K/V heads, D 128 causal: the same bits as the per-head runner given each K/V head repeated 4x
    const int64_t B = 2, H = 8, Hkv = 2, S = 300, D = 128, g = H / Hkv;
    const size_t nq = prod({B, H, S, D}), nkv = prod({B, Hkv, S, D});
    auto qq = to_bf16(normal(nq, 20)), kq = to_bf16(normal(nkv, 21)), vq = to_bf16(normal(nkv, 22));
    std::vector<uint16_t> kx(nq), vx(nq);
    for (int64_t b = 0; b < B; ++b)
        for (int64_t h = 0; h < H; ++h)
            for (int64_t e = 0; e < S * D; ++e) {
                kx[((b * H + h) * S * D) + e] = kq[((b * Hkv + h / g) * S * D) + e];
                vx[((b * H + h) * S * D) + e] = vq[((b * Hkv + h / g) * S * D) + e];
            }
    const float sc = default_scale(D);
    DeviceMemory dq = upload(qq), dk = upload(kq), dv = upload(vq), dkx = upload(kx), dvx = upload(vx);
    DeviceMemory o1(nq * 2), o2(nq * 2), l1(B * H * S * 4), l2(B * H * S * 4);
    harness::flash_attention_fwd_fused::run_flash_attention_fwd_fused_gqa_device(
        dq.data(), dk.data(), dv.data(), o1.data(), l1.as<float>(), B, H, Hkv, S, S, D, D, sc, 1, Dtype::BF16);
    harness::flash_attention_fwd_fused::run_flash_attention_fwd_fused_device(
        dq.data(), dkx.data(), dvx.data(), o2.data(), l2.as<float>(), B, H, S, S, D, D, sc, 1, Dtype::BF16);
    ASSERT_TRUE(harness::device::DeviceSynchronize());
    ASSERT_TRUE(harness::device::CheckDeviceError());
    EXPECT_TRUE(download<uint16_t>(o1, nq) == download<uint16_t>(o2, nq)) << "O bit-identical";
    EXPECT_TRUE(download<float>(l1, B * H * S) == download<float>(l2, B * H * S)) << "lse bit-identical";
}

TEST(FlashAttentionTest, HostBufferRunnerMatchesDevice) {
    const int64_t B = 2, H = 5, S = 700, D = 128;
    const size_t n = prod({B, H, S, D});
    auto qq = to_bf16(normal(n, 10)), kq = to_bf16(normal(n, 11)), vq = to_bf16(normal(n, 12));
    const float sc = default_scale(D);
    std::vector<uint16_t> ho(n);
    std::vector<float> hl(B * H * S);
    harness::flash_attention_fwd_fused::run_flash_attention_fwd_fused_host(qq.data(), kq.data(), vq.data(), ho.data(),
                                                                           hl.data(), B, H, S, S, D, D, sc, 1,
                                                                           Dtype::BF16);
    DeviceMemory dq = upload(qq), dk = upload(kq), dv = upload(vq), dout(n * 2), dlse(B * H * S * 4);
    harness::flash_attention_fwd_fused::run_flash_attention_fwd_fused_device(
        dq.data(), dk.data(), dv.data(), dout.data(), dlse.as<float>(), B, H, S, S, D, D, sc, 1, Dtype::BF16);
    ASSERT_TRUE(harness::device::DeviceSynchronize());
    EXPECT_TRUE(download<uint16_t>(dout, n) == ho) << "O bit-identical";
    EXPECT_TRUE(download<float>(dlse, B * H * S) == hl) << "lse bit-identical";
}

MINI_GTEST_MAIN
