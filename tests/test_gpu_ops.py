"""GPU parity of the bandwidth-bound ladder operators against the pinned CPU oracle.

For every case of the reference's GTest suites (tests/cases.py) the CUDA kernel, called through
the C ABI, is compared with the oracle on the same inputs: bit-exact for elementwise add, axpy,
broadcast and transposes (fp32 and 16-bit), and within the reference's tolerances otherwise
(activation 1e-5, reduce 1e-4, layer_norm / rms_norm_rope 1e-4 in fp32).  The benchmarked
configurations run at full size with their stated tolerances (layer_norm max-abs 1e-2,
rms_norm_rope max-abs 2e-2, elementwise_add bit-exact); for 16-bit outputs an element also passes
when it is within half an output ulp (relative) of the fp32 golden, because above |y| = 2.56
(bf16) a single correct rounding of the output already exceeds 1e-2."""
from __future__ import annotations

import numpy as np
import pytest

import cases as C
import specs
from accuracy import assert_close
from gpu_util import bits, dev, host, quantize

pytestmark = pytest.mark.gpu

KINDS = ["f32", "bf16", "f16"]
# Half a unit in the last place, relative, of a correctly rounded 16-bit output.
OUT_HALF_ULP = {"bf16": 2.0 ** -8, "f16": 2.0 ** -11}


# --------------------------------------------------------------------------- elementwise_add
@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("shape", C.ELEMENTWISE_SHAPES + [(4097,), (0,)], ids=lambda s: "x".join(map(str, s)) or "empty")
def test_elementwise_add(cuda, hc_lib, oracle, shape, kind):
    n = int(np.prod(shape))
    x = oracle.uniform(n, C.SEED).reshape(shape)
    y = oracle.uniform(n, C.SEED + 1).reshape(shape)
    z = hc_lib.elementwise_add(dev(x, kind, oracle), dev(y, kind, oracle))
    ref = oracle.elementwise_add(quantize(x, kind, oracle), quantize(y, kind, oracle))
    if kind == "f32":
        assert np.array_equal(host(z, oracle), ref)
    else:
        enc = oracle.to_bf16(ref) if kind == "bf16" else oracle.to_f16(ref)
        assert np.array_equal(bits(z), enc.reshape(z.shape))


def test_elementwise_add_config_bit_exact(cuda, hc_lib, oracle):
    """Benchmarked configuration: fp16 [4096, 8192], x ~ U[-1,1] seed 0, y seed 1, bit-exact."""
    shape = tuple(specs.bench_config("elementwise_add")["shape"])  # (4096, 8192)
    n = int(np.prod(shape))
    x = oracle.uniform(n, 0).reshape(shape)
    y = oracle.uniform(n, 1).reshape(shape)
    z = hc_lib.elementwise_add(dev(x, "f16", oracle), dev(y, "f16", oracle))
    ref = oracle.to_f16(oracle.elementwise_add(quantize(x, "f16", oracle), quantize(y, "f16", oracle)))
    assert np.array_equal(bits(z), ref)


def test_elementwise_add_unaligned_views(cuda, hc_lib, oracle):
    """Buffers that are not 16-byte aligned take the scalar kernel and stay bit-exact."""
    import torch

    base = oracle.uniform(1001, 5)
    t = dev(base, "f16", oracle)
    x, y = t[1:1000], t[:999]
    out = torch.empty(1000, dtype=torch.float16, device="cuda")[1:]
    hc_lib.elementwise_add(x, y, out)
    q = quantize(base, "f16", oracle)
    assert np.array_equal(bits(out), oracle.to_f16(oracle.elementwise_add(q[1:1000], q[:999])))


# --------------------------------------------------------------------------- axpy
@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("case", C.AXPY_CASES, ids=lambda c: "{}_{}_{}".format("x".join(map(str, c[0])), c[1], c[2]))
def test_axpy(cuda, hc_lib, oracle, case, kind):
    shape, a, b = case
    x = oracle.uniform(int(np.prod(shape)), C.SEED).reshape(shape)
    y = hc_lib.axpy_scalar_affine(dev(x, kind, oracle), a, b)
    ref = oracle.axpy_scalar_affine(quantize(x, kind, oracle), a, b)
    if kind == "f32":
        assert np.array_equal(host(y, oracle), ref)
    else:
        assert np.array_equal(bits(y), (oracle.to_bf16(ref) if kind == "bf16" else oracle.to_f16(ref)).reshape(y.shape))


# --------------------------------------------------------------------------- broadcast_binary
@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("case", C.BROADCAST_CASES, ids=lambda c: "B{}_C{}_H{}_W{}_yb{}".format(*c))
def test_broadcast_binary(cuda, hc_lib, oracle, case, kind):
    B, Cc, H, W, yb = case
    x = oracle.uniform(B * Cc * H * W, C.SEED).reshape(B, Cc, H, W)
    y = oracle.uniform(yb * Cc, C.SEED + 1)
    bias = oracle.uniform(Cc, C.SEED + 2)
    z = hc_lib.broadcast_binary(dev(x, kind, oracle), dev(y, kind, oracle), dev(bias, kind, oracle), yb)
    ref = oracle.broadcast_binary(quantize(x, kind, oracle), quantize(y, kind, oracle), quantize(bias, kind, oracle), yb)
    if kind == "f32":
        assert np.array_equal(host(z, oracle), ref)
    else:
        assert np.array_equal(bits(z), oracle.to_bf16(ref) if kind == "bf16" else oracle.to_f16(ref))


# --------------------------------------------------------------------------- activation
@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("case", C.ACTIVATION_CASES + [((1 << 20,), "gelu"), ((1 << 20,), "silu")],
                         ids=lambda c: "{}_{}".format("x".join(map(str, c[0])), c[1]))
def test_activation(cuda, hc_lib, oracle, case, kind):
    shape, act = case
    x = oracle.uniform(int(np.prod(shape)), C.SEED, -8.0, 8.0).reshape(shape)
    y = hc_lib.activation_gelu_silu(dev(x, kind, oracle), act)
    ref = oracle.activation_gelu_silu(quantize(x, kind, oracle), act)
    if kind == "f32":
        assert_close(ref, host(y, oracle), 1e-5, 1e-5, f"{act} f32")  # test_activation_gelu_silu.cpp:59
    else:
        # one rounding of an fp32 value within 1e-5 of the golden: at most one 16-bit ulp apart
        ulp = 2.0 ** -7 if kind == "bf16" else 2.0 ** -10
        assert_close(quantize(ref, kind, oracle), host(y, oracle), 1e-5, ulp, f"{act} {kind}")


def test_activation_spec_values(cuda, hc_lib, oracle):
    x = np.array(C.ACTIVATION_SPEC_VALUES, np.float32)
    for act in ("gelu", "silu"):
        y = host(hc_lib.activation_gelu_silu(dev(x, "f32", oracle), act), oracle)
        assert_close(oracle.activation_gelu_silu(x, act), y, 1e-5, 1e-5, act)


# --------------------------------------------------------------------------- reduce_sum_lastdim
@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("case", C.REDUCE_CASES + [(1, 2, 100000), (1, 16384, 4096)], ids=lambda c: "B{}_M{}_K{}".format(*c))
def test_reduce_sum(cuda, hc_lib, oracle, case, kind):
    B, M, K = case
    x = oracle.uniform(B * M * K, C.SEED).reshape(B, M, K)
    out = hc_lib.reduce_sum_lastdim(dev(x, kind, oracle))
    ref = oracle.reduce_sum_lastdim(quantize(x, kind, oracle).reshape(B * M, K)).reshape(B, M)
    assert_close(ref, host(out, oracle), 1e-4, 1e-4, f"reduce {case}")  # test_reduce_sum_lastdim.cpp:16


def test_reduce_sum_known_answers(cuda, hc_lib, oracle):
    out = host(hc_lib.reduce_sum_lastdim(dev(np.array([[1, 2, 3], [4, 5, 6]], np.float32), "f32", oracle)), oracle)
    assert out.tolist() == [6.0, 15.0]
    ones = host(hc_lib.reduce_sum_lastdim(dev(np.ones((1, 100000), np.float32), "f32", oracle)), oracle)
    assert abs(ones[0] - 100000.0) <= 1.0


# --------------------------------------------------------------------------- transpose
@pytest.mark.parametrize("dtype", ["f32", "i32", "bf16", "u8"])
@pytest.mark.parametrize("case", C.TRANSPOSE_2D_CASES + [(4096, 4100)], ids=lambda c: "{}x{}".format(*c))
def test_transpose_2d(cuda, hc_lib, oracle, case, dtype):
    import torch

    M, N = case
    if dtype == "f32":
        x = torch.from_numpy(oracle.uniform(M * N, C.SEED).reshape(M, N)).cuda()
    elif dtype == "i32":
        x = torch.from_numpy((np.arange(M * N, dtype=np.int32) * 7 - 3).reshape(M, N)).cuda()
    elif dtype == "bf16":
        x = dev(oracle.uniform(M * N, C.SEED).reshape(M, N), "bf16", oracle)
    else:
        x = torch.from_numpy((np.arange(M * N) % 251).astype(np.uint8).reshape(M, N)).cuda()
    y = hc_lib.transpose_2d_4d(x, 0)
    assert torch.equal(y.cpu(), x.cpu().t().contiguous())


@pytest.mark.parametrize("case", C.TRANSPOSE_4D_CASES, ids=lambda c: "{}x{}x{}x{}".format(*c))
def test_transpose_4d_and_round_trip(cuda, hc_lib, oracle, case):
    import torch

    n, c, h, w = case
    xf = oracle.uniform(n * c * h * w, C.SEED).reshape(n, c, h, w)
    x = torch.from_numpy(xf).cuda()
    y = hc_lib.transpose_2d_4d(x, 1)
    assert np.array_equal(y.cpu().numpy(), oracle.transpose(xf, 1))
    back = hc_lib.transpose_2d_4d(y, 2)
    assert torch.equal(back, x)
    xi = torch.from_numpy((np.arange(n * c * h * w, dtype=np.int32) - 5).reshape(n, h, w, c)).cuda()
    assert np.array_equal(hc_lib.transpose_2d_4d(xi, 2).cpu().numpy(), oracle.transpose(xi.cpu().numpy(), 2))


# --------------------------------------------------------------------------- layer_norm
@pytest.mark.parametrize("case", C.LAYER_NORM_CASES + [(3, 100, 1e-5), (2, 40000, 1e-5)], ids=lambda c: "rows{}_dim{}_eps{}".format(*c))
def test_layer_norm_f32(cuda, hc_lib, oracle, case):
    rows, dim, eps = case
    x, g, b = C.layer_norm_inputs(oracle, rows, dim)
    y = hc_lib.layer_norm(dev(x, "f32", oracle), dev(g, "f32", oracle), dev(b, "f32", oracle), eps)
    assert_close(oracle.layer_norm(x, g, b, eps), host(y, oracle), 1e-4, 1e-4, f"layer_norm {case}")  # test_layer_norm.cpp:33


def test_layer_norm_constant_row(cuda, hc_lib, oracle):
    g = oracle.uniform(128, 99, 0.5, 1.5)
    b = oracle.uniform(128, 100, -0.5, 0.5)
    y = hc_lib.layer_norm(dev(np.full((4, 128), 3.5, np.float32), "f32", oracle), dev(g, "f32", oracle),
                          dev(b, "f32", oracle), 1e-5)
    np.testing.assert_allclose(host(y, oracle), np.broadcast_to(b, (4, 128)), atol=1e-4)


@pytest.mark.parametrize("kind", ["bf16", "f16"])
def test_layer_norm_config(cuda, hc_lib, oracle, kind):
    """Benchmarked configuration: bf16 [16384, 4096], x ~ N(0,1) seed 0, gamma ~ U[0.5,1.5], beta ~ U[-0.1,0.1],
    eps 1e-5, max-abs 1e-2 (checked on every row)."""
    cfg = specs.bench_config("layer_norm")
    rows, dim = cfg["rows"], cfg["lastDim"]
    x = oracle.normal(rows * dim, 0).reshape(rows, dim)
    g = oracle.uniform(dim, 1, 0.5, 1.5)
    b = oracle.uniform(dim, 2, -0.1, 0.1)
    y = hc_lib.layer_norm(dev(x, kind, oracle), dev(g, "f32", oracle), dev(b, "f32", oracle), 1e-5)
    ref = oracle.layer_norm(quantize(x, kind, oracle), g, b, 1e-5)
    # max-abs 1e-2, or (where |y| is so large that one 16-bit rounding alone exceeds 1e-2) half an
    # output ulp relative: CompareArrays semantics, an element fails only if both are exceeded.
    assert_close(ref, host(y, oracle), 1e-2, OUT_HALF_ULP[kind], "layer_norm config")


# --------------------------------------------------------------------------- rms_norm_rope_fused
@pytest.mark.parametrize("case", C.RMS_ROPE_CASES, ids=lambda c: "B{}_S{}_H{}_rot{}_eps{}".format(*c))
def test_rms_norm_rope_reference_layout(cuda, hc_lib, oracle, case):
    """The golden's own layout [B, S, H] with interleaved pairs."""
    B, S, H, rot, eps = case
    x, w, cos, sin = C.rms_rope_inputs(oracle, B, S, H, rot)
    out = hc_lib.rms_norm_rope_fused(dev(x, "f32", oracle), dev(w, "f32", oracle), dev(cos, "f32", oracle),
                                     dev(sin, "f32", oracle), rot, eps)
    ref = oracle.rms_norm_rope(x, w, cos, sin, rot, eps)
    assert_close(ref, host(out, oracle), 1e-4, 1e-4, f"rms_norm_rope {case}")  # test_rms_norm_rope_fused.cpp:37


@pytest.mark.parametrize("style", [0, 1])
@pytest.mark.parametrize("H,rot", [(128, 128), (128, 64), (64, 32), (256, 128), (40, 24)])
def test_rms_norm_rope_heads_and_styles(cuda, hc_lib, oracle, style, H, rot):
    B, S, Hh = 2, 33, 3
    x = oracle.normal(B * S * Hh * H, 3).reshape(B, S, Hh, H)
    w = oracle.uniform(H, 4, 0.5, 1.5)
    cos, sin = oracle.rope_cos_sin(S, rot // 2)
    for kind, tol in (("f32", 1e-4), ("bf16", 2e-2)):
        out = hc_lib.rms_norm_rope_fused(dev(x, kind, oracle), dev(w, "f32", oracle), dev(cos, "f32", oracle),
                                         dev(sin, "f32", oracle), rot, 1e-6, heads=Hh, rope_style=style)
        ref = oracle.rms_norm_rope(quantize(x, kind, oracle), w, cos, sin, rot, 1e-6, heads=Hh, style=style)
        assert_close(ref, host(out, oracle), tol, 1e-4 if kind == "f32" else OUT_HALF_ULP[kind], f"{kind} style{style}")


def test_rms_norm_rope_config(cuda, hc_lib, oracle):
    """Benchmarked configuration: x bf16 [8, 4096, 32, 128] ~ N(0,1) seed 0, weight ~ U[0.5,1.5], eps 1e-6,
    rotate-half RoPE theta 10000, fp32 cos/sin; max-abs 2e-2 on every element."""
    cfg = specs.bench_config("rms_norm_rope_fused")
    B, S, Hh, D = cfg["B"], cfg["S"], cfg["heads"], cfg["H"]
    x = oracle.normal(B * S * Hh * D, 0).reshape(B, S, Hh, D)
    w = oracle.uniform(D, 1, 0.5, 1.5)
    cos, sin = oracle.rope_cos_sin(S, D // 2, 10000.0)
    out = hc_lib.rms_norm_rope_fused(dev(x, "bf16", oracle), dev(w, "f32", oracle), dev(cos, "f32", oracle),
                                     dev(sin, "f32", oracle), D, 1e-6, heads=Hh, rope_style=1)
    got = host(out, oracle)
    del out
    for b in range(B):  # oracle per batch keeps host memory bounded
        ref = oracle.rms_norm_rope(quantize(x[b:b + 1], "bf16", oracle), w, cos, sin, D, 1e-6, heads=Hh, style=1)
        assert_close(ref, got[b:b + 1], 2e-2, OUT_HALF_ULP["bf16"], f"rms_norm_rope config batch {b}")


# --------------------------------------------------------------------------- unrolled row paths
@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("dim", [256, 512, 1024, 2048, 4096])
def test_layer_norm_unrolled_widths(cuda, hc_lib, oracle, kind, dim):
    """Rows of exactly 32*KPL packs take the unrolled LayerNorm (KPL 2..16); others the generic loop."""
    rows = 37
    x = oracle.normal(rows * dim, 11).reshape(rows, dim) * 2.0 + 0.5
    g = oracle.uniform(dim, 12, 0.5, 1.5)
    b = oracle.uniform(dim, 13, -0.1, 0.1)
    y = hc_lib.layer_norm(dev(x, kind, oracle), dev(g, "f32", oracle), dev(b, "f32", oracle), 1e-5)
    ref = oracle.layer_norm(quantize(x, kind, oracle), g, b, 1e-5)
    if kind == "f32":
        assert_close(ref, host(y, oracle), 1e-4, 1e-4, f"layer_norm f32 dim {dim}")
    else:
        assert_close(ref, host(y, oracle), 1e-2, OUT_HALF_ULP[kind], f"layer_norm {kind} dim {dim}")


@pytest.mark.parametrize("dim", [64, 256, 1024, 4096])
def test_layer_norm_reference_low_variance_row(cuda, hc_lib, oracle, dim):
    """test_layer_norm.cpp:91-117: rows base + 1e-6 * d (base 5 and -3), gamma/beta seeds 101/102,
    tolerance 1e-4 -- at the reference's dim 64 and at widths that take the unrolled paths."""
    x = np.stack([np.float32(base) + np.float32(1e-6) * np.arange(dim, dtype=np.float32) for base in (5.0, -3.0)])
    g = oracle.uniform(dim, 101, 0.5, 1.5)
    b = oracle.uniform(dim, 102, -0.5, 0.5)
    y = hc_lib.layer_norm(dev(x, "f32", oracle), dev(g, "f32", oracle), dev(b, "f32", oracle), 1e-5)
    assert_close(oracle.layer_norm(x, g, b, 1e-5), host(y, oracle), 1e-4, 1e-4, f"low variance dim {dim}")


def test_layer_norm_low_variance_rows(cuda, hc_lib, oracle):
    """Large mean, tiny spread (test_layer_norm.cpp:92-117 style): the centred passes keep it accurate."""
    rows, dim = 8, 1024
    x = (1000.0 + oracle.uniform(rows * dim, 21, -1e-2, 1e-2)).astype(np.float32).reshape(rows, dim)
    g = np.ones(dim, np.float32)
    b = np.zeros(dim, np.float32)
    y = hc_lib.layer_norm(dev(x, "f32", oracle), dev(g, "f32", oracle), dev(b, "f32", oracle), 1e-5)
    assert_close(oracle.layer_norm(x, g, b, 1e-5), host(y, oracle), 2e-3, 2e-3, "low variance")


@pytest.mark.parametrize("kind", KINDS)
def test_rms_norm_rope_lane_local_and_unaligned_weight(cuda, hc_lib, oracle, kind):
    """Rotate-half over the whole row (the lane-local fast path), and the same call with a weight
    vector that is not 16-byte aligned, which must take the generic path with the same results."""
    B, S, Hh, H = 3, 65, 4, 128
    x = oracle.normal(B * S * Hh * H, 31).reshape(B, S, Hh, H)
    w = oracle.uniform(H + 1, 32, 0.5, 1.5)
    cos, sin = oracle.rope_cos_sin(S, H // 2)
    wd = dev(w, "f32", oracle)
    xd, cd, sd = dev(x, kind, oracle), dev(cos, "f32", oracle), dev(sin, "f32", oracle)
    tol = (1e-4, 1e-4) if kind == "f32" else (2e-2, OUT_HALF_ULP[kind])
    for off in (0, 1):
        wv = wd[off:off + H]
        assert wv.data_ptr() % 16 == 4 * off
        out = hc_lib.rms_norm_rope_fused(xd, wv, cd, sd, H, 1e-6, heads=Hh, rope_style=1)
        ref = oracle.rms_norm_rope(quantize(x, kind, oracle), w[off:off + H], cos, sin, H, 1e-6, heads=Hh, style=1)
        assert_close(ref, host(out, oracle), *tol, f"{kind} weight offset {off}")


@pytest.mark.parametrize("kind", ["f32", "bf16"])
@pytest.mark.parametrize("dim", [1024, 2048, 4096])
def test_layer_norm_outlier_first_element(cuda, hc_lib, oracle, kind, dim):
    """Rows whose first element is far from the mean: the one-pass shifted variance of the
    group-per-row kernel must fall back to the exact centred pass (alternate rows do)."""
    rows = 6
    x = oracle.normal(rows * dim, 41).reshape(rows, dim)
    x[::2, 0] = 1000.0
    x[1::2, 0] = -250.0
    g = oracle.uniform(dim, 42, 0.5, 1.5)
    b = oracle.uniform(dim, 43, -0.1, 0.1)
    y = hc_lib.layer_norm(dev(x, kind, oracle), dev(g, "f32", oracle), dev(b, "f32", oracle), 1e-5)
    ref = oracle.layer_norm(quantize(x, kind, oracle), g, b, 1e-5)
    if kind == "f32":
        assert_close(ref, host(y, oracle), 1e-4, 1e-4, f"outlier f32 dim {dim}")
    else:
        assert_close(ref, host(y, oracle), 1e-2, OUT_HALF_ULP[kind], f"outlier bf16 dim {dim}")


@pytest.mark.parametrize("case", C.TRANSPOSE_4D_CASES + [(2, 64, 56, 56), (3, 5, 7, 9)],
                         ids=lambda c: "{}x{}x{}x{}".format(*c))
def test_transpose_4d_16bit_round_trip(cuda, hc_lib, oracle, case):
    """2-byte elements: extents that are not multiples of 8 take the 64x64 register-tile kernel (odd extents
    exercise its edge and misaligned-word paths); the others take the TMA-fed kernel."""
    n, c, h, w = case
    xf = oracle.uniform(n * c * h * w, C.SEED).reshape(n, c, h, w)
    x = dev(xf, "bf16", oracle)
    y = hc_lib.transpose_2d_4d(x, 1)
    assert np.array_equal(bits(y), oracle.transpose(bits(x), 1))
    assert np.array_equal(bits(hc_lib.transpose_2d_4d(y, 2)), bits(x))


@pytest.mark.parametrize("case", [(8, 8), (264, 72), (520, 200), (1024, 4096), (4104, 8), (8, 4104)],
                         ids=lambda c: "{}x{}".format(*c))
def test_transpose_16bit_tma_tiles(cuda, hc_lib, oracle, case):
    """Extents that are multiples of 8 take the TMA-fed kernel (256 x 64 tiles): partial tiles at both
    edges, and more tiles than resident blocks.  An offset view (not 16-byte aligned) of the same
    data takes the register-tile kernel and must give the same bits."""
    import torch

    M, N = case
    xi = torch.from_numpy((np.arange(M * N, dtype=np.int64) % 65521).astype(np.int16).reshape(M, N)).cuda()
    want = xi.cpu().t().contiguous()
    y = hc_lib.transpose_2d_4d(xi.view(torch.bfloat16), 0)
    assert torch.equal(y.view(torch.int16).cpu(), want)
    # two elements in: 4-byte aligned (register-tile kernel), not 16-byte aligned (no TMA)
    buf = torch.empty(M * N + 2, dtype=torch.int16, device="cuda")
    buf[2:].copy_(xi.reshape(-1))
    xo = buf[2:].view(M, N).view(torch.bfloat16)
    assert torch.equal(hc_lib.transpose_2d_4d(xo, 0).view(torch.int16).cpu(), want)


@pytest.mark.parametrize("case", [(3, 24, 17, 8), (2, 8, 64, 48)], ids=lambda c: "{}x{}x{}x{}".format(*c))
def test_transpose_4d_16bit_tma_round_trip(cuda, hc_lib, oracle, case):
    """Batched NCHW <-> NHWC with channel and plane sizes that are multiples of 8 (TMA-fed kernel)."""
    n, c, h, w = case
    xf = oracle.uniform(n * c * h * w, C.SEED).reshape(n, c, h, w)
    x = dev(xf, "bf16", oracle)
    y = hc_lib.transpose_2d_4d(x, 1)
    assert np.array_equal(bits(y), oracle.transpose(bits(x), 1))
    assert np.array_equal(bits(hc_lib.transpose_2d_4d(y, 2)), bits(x))
