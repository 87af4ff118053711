"""Pins the CPU oracle to the reference harness: bit-identical outputs on every case of the
reference's own GTest suites (fixtures produced by the reference goldens themselves, see
tests/golden/make_golden.py), plus the reference tests' hand-computed known answers.
CPU only."""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

import cases as C

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "reference_goldens.json").read_text())


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def assert_pinned(group: str, key: str, out: np.ndarray):
    ref = GOLDEN[group][key]
    assert list(out.shape) == ref["shape"], (group, key)
    assert sha(out) == ref["sha256"], f"{group}/{key}: oracle {out.reshape(-1)[:6]} vs reference {ref['head']}"


def test_generator_pinned(oracle):
    for seed, lo, hi, n in [(C.SEED, -1.0, 1.0, 4096), (C.SEED + 1000, -1.0, 1.0, 4096), (C.SEED, -3.0, 3.0, 4096),
                            (C.SEED + 1, 0.5, 1.5, 4096), (C.SEED, -2.0, 2.0, 4096), (0, -1.0, 1.0, 4096)]:
        assert_pinned("generator", f"uniform_{seed}_{lo}_{hi}_{n}", oracle.uniform(n, seed, lo, hi))
    for S, half in [(16, 32), (128, 32), (4096, 64)]:
        c, s = oracle.rope_cos_sin(S, half)
        ref = GOLDEN["generator"][f"rope_{S}_{half}"]
        assert sha(c) == ref["cos"]["sha256"] and sha(s) == ref["sin"]["sha256"]


@pytest.mark.parametrize("case", C.FA_CASES, ids=lambda c: "B{}_H{}_Sq{}_Sk{}_D{}_Dv{}_{}".format(*c[:6], "causal" if c[6] else "none"))
def test_flash_attention_pinned(oracle, case):
    B, H, Sq, Sk, D, Dv, causal = case
    q, k, v = C.fa_inputs(oracle, B, H, Sq, Sk, D, Dv)
    o, lse = oracle.flash_attention_fwd(q, k, v, C.default_scale(D), causal)
    assert_pinned("flash_attention", "_".join(map(str, case)), o)
    assert np.all(np.isfinite(lse))


def test_flash_attention_special_pinned(oracle):
    from golden.make_golden import special_fa_inputs

    q = oracle.uniform(2 * 8 * 32, 99).reshape(1, 2, 8, 32)
    k = oracle.uniform(2 * 8 * 32, 100).reshape(1, 2, 8, 32)
    v = oracle.uniform(2 * 8 * 32, 101).reshape(1, 2, 8, 32)
    base = np.float32(1.0) / np.sqrt(np.float32(32))
    o1, _ = oracle.flash_attention_fwd(q, k, v, float(base), 0)
    o2, _ = oracle.flash_attention_fwd(q, (k * np.float32(2)).astype(np.float32), v, float(base / np.float32(2)), 0)
    assert_pinned("flash_attention_special", "scale_invariance_base", o1)
    assert_pinned("flash_attention_special", "scale_invariance_2k", o2)
    np.testing.assert_allclose(o1, o2, atol=1e-4, rtol=1e-4)  # test_flash_attention_fwd_fused.cpp:252-254
    for name, (q, k, v, sc, causal) in special_fa_inputs().items():
        o, _ = oracle.flash_attention_fwd(q, k, v, float(sc), causal)
        assert_pinned("flash_attention_special", name, o)
        if name == "causal_constraint":  # :213-223
            col = o[0, 0, :, 0]
            assert np.all(col >= 0.0) and np.all(col <= np.arange(8) + 0.01)
        else:  # :277-288
            np.testing.assert_allclose(o[0, 0, :, 0], 1.0, atol=1e-4)
            np.testing.assert_allclose(o[0, 0, :, 1:], 0.0, atol=1e-4)


def test_flash_attention_lse_definition(oracle):
    """lse (no reference counterpart) = log(sum_j exp(scale*q.k_j)) over visible keys, fp64 check."""
    q, k, v = C.fa_inputs(oracle, 1, 2, 40, 40, 32, 32)
    for causal in (0, 1):
        _, lse = oracle.flash_attention_fwd(q, k, v, 0.2, causal)
        s = np.einsum("bhqd,bhkd->bhqk", q.astype(np.float64), k.astype(np.float64)) * np.float64(np.float32(0.2))
        if causal:
            s = np.where(np.triu(np.ones((40, 40), bool), 1), -np.inf, s)
        m = s.max(-1, keepdims=True)
        ref = (m[..., 0] + np.log(np.exp(s - m).sum(-1)))
        np.testing.assert_allclose(lse, ref, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("shape", [(1, 2, 37, 37, 16, 16), (2, 1, 20, 45, 8, 12), (1, 1, 45, 20, 12, 8)])
@pytest.mark.parametrize("causal", [0, 1])
def test_flash_attention_bwd_against_autograd(oracle, shape, causal):
    """The backward oracle (no reference counterpart: the ladder is forward only) against torch
    float64 autograd of the same forward, top-left causal mask as the reference golden."""
    import torch

    B, H, S_q, S_k, D, Dv = shape
    q, k, v = C.fa_inputs(oracle, B, H, S_q, S_k, D, Dv)
    do = oracle.uniform(B * H * S_q * Dv, 99).reshape(B, H, S_q, Dv)
    scale = 0.3
    dq, dk, dv = oracle.flash_attention_bwd(q, k, v, do, scale, causal)
    tq, tk, tv = (torch.tensor(a, dtype=torch.float64, requires_grad=True) for a in (q, k, v))
    s = tq @ tk.transpose(-1, -2) * float(np.float32(scale))
    if causal:
        s = s.masked_fill(torch.ones(S_q, S_k, dtype=torch.bool).triu(1), float("-inf"))
    (torch.softmax(s, -1) @ tv).backward(torch.tensor(do, dtype=torch.float64))
    for got, ref in ((dq, tq.grad), (dk, tk.grad), (dv, tv.grad)):
        np.testing.assert_allclose(got, ref.numpy(), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("case", C.MATMUL_CASES, ids=lambda c: "M{}_K{}_N{}_{}".format(c[0], c[1], c[2], "bias" if c[3] else "nobias"))
def test_matmul_bias_pinned(oracle, case):
    M, K, N, wb = case
    A, B, bias = C.matmul_inputs(oracle, M, K, N)
    assert_pinned("matmul_bias", f"{M}_{K}_{N}_{int(wb)}", oracle.matmul_bias(A, B, bias if wb else None))


def test_matmul_identity(oracle):
    """test_matmul_bias.cpp:71-94: A . I = A."""
    A = oracle.uniform(64 * 64, 7, -2, 2).reshape(64, 64)
    np.testing.assert_allclose(oracle.matmul_bias(A, np.eye(64, dtype=np.float32)), A, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("case", C.LAYER_NORM_CASES, ids=lambda c: "rows{}_dim{}_eps{}".format(*c))
def test_layer_norm_pinned(oracle, case):
    rows, dim, eps = case
    x, g, b = C.layer_norm_inputs(oracle, rows, dim)
    assert_pinned("layer_norm", f"{rows}_{dim}_{eps}", oracle.layer_norm(x, g, b, eps))


def test_layer_norm_constant_and_low_variance(oracle):
    """test_layer_norm.cpp:61-117: a constant row gives beta; near-constant rows stay finite."""
    g = oracle.uniform(128, 99, 0.5, 1.5)
    b = oracle.uniform(128, 100, -0.5, 0.5)
    y = oracle.layer_norm(np.full((4, 128), 3.5, np.float32), g, b, 1e-5)
    np.testing.assert_allclose(y, np.broadcast_to(b, y.shape), atol=1e-4)
    x = np.stack([5.0 + 1e-6 * np.arange(64), -3.0 + 1e-6 * np.arange(64)]).astype(np.float32)
    assert np.all(np.isfinite(oracle.layer_norm(x, g[:64], b[:64], 1e-5)))


@pytest.mark.parametrize("case", C.RMS_ROPE_CASES, ids=lambda c: "B{}_S{}_H{}_rot{}_eps{}".format(*c))
def test_rms_norm_rope_pinned(oracle, case):
    B, S, H, rot, eps = case
    x, w, cos, sin = C.rms_rope_inputs(oracle, B, S, H, rot)
    assert_pinned("rms_norm_rope_fused", f"{B}_{S}_{H}_{rot}_{eps}", oracle.rms_norm_rope(x, w, cos, sin, rot, eps))


def test_rope_rotate_half_is_permuted_interleaved(oracle):
    """The rotate-half variant equals the golden's interleaved form under the pairing permutation
    pi(2d) = d, pi(2d+1) = d + half (how the config's rotate-half RoPE maps onto the golden)."""
    B, S, Hh, D = 2, 8, 3, 128
    x = oracle.normal(B * S * Hh * D, 0).reshape(B, S, Hh, D)
    w = oracle.uniform(D, 1, 0.5, 1.5)
    cos, sin = oracle.rope_cos_sin(S, D // 2)
    out_rh = oracle.rms_norm_rope(x, w, cos, sin, D, 1e-6, heads=Hh, style=1)
    perm = np.empty(D, np.int64)
    perm[0::2] = np.arange(D // 2)
    perm[1::2] = np.arange(D // 2) + D // 2
    xi = x[..., perm]
    cos_rows = np.repeat(cos, Hh, axis=0).reshape(S * Hh, D // 2)
    sin_rows = np.repeat(sin, Hh, axis=0).reshape(S * Hh, D // 2)
    out_il = oracle.rms_norm_rope(xi.reshape(B, S * Hh, D), w[perm], cos_rows, sin_rows, D, 1e-6)
    back = np.empty_like(out_il)
    back[..., perm] = out_il
    np.testing.assert_allclose(out_rh.reshape(B, S * Hh, D), back, rtol=2e-6, atol=2e-6)


@pytest.mark.parametrize("shape", C.ELEMENTWISE_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_elementwise_add_pinned(oracle, shape):
    n = int(np.prod(shape))
    assert_pinned("elementwise_add", "x".join(map(str, shape)),
                  oracle.elementwise_add(oracle.uniform(n, C.SEED), oracle.uniform(n, C.SEED + 1)))


def test_elementwise_add_hand_values(oracle):
    z = oracle.elementwise_add(np.array([1, 2, 3, 4], np.float32), np.array([5, 6, 7, 8], np.float32))
    assert_pinned("elementwise_add", "hand_1234_5678", z)
    assert z.tolist() == [6.0, 8.0, 10.0, 12.0]  # test_elementwise_add.cpp:19-28


@pytest.mark.parametrize("case", C.AXPY_CASES, ids=lambda c: "{}_{}_{}".format("x".join(map(str, c[0])), c[1], c[2]))
def test_axpy_pinned(oracle, case):
    shape, a, b = case
    n = int(np.prod(shape))
    assert_pinned("axpy_scalar_affine", f"{'x'.join(map(str, shape))}_{a}_{b}",
                  oracle.axpy_scalar_affine(oracle.uniform(n, C.SEED), a, b))


@pytest.mark.parametrize("case", C.BROADCAST_CASES, ids=lambda c: "B{}_C{}_H{}_W{}_yb{}".format(*c))
def test_broadcast_binary_pinned(oracle, case):
    B, Cc, H, W, yb = case
    x = oracle.uniform(B * Cc * H * W, C.SEED).reshape(B, Cc, H, W)
    y = oracle.uniform(yb * Cc, C.SEED + 1)
    bias = oracle.uniform(Cc, C.SEED + 2)
    assert_pinned("broadcast_binary", f"{B}_{Cc}_{H}_{W}_{yb}", oracle.broadcast_binary(x, y, bias, yb))


@pytest.mark.parametrize("case", C.ACTIVATION_CASES, ids=lambda c: "{}_{}".format("x".join(map(str, c[0])), c[1]))
def test_activation_pinned(oracle, case):
    shape, act = case
    n = int(np.prod(shape))
    assert_pinned("activation_gelu_silu", f"{'x'.join(map(str, shape))}_{act}",
                  oracle.activation_gelu_silu(oracle.uniform(n, C.SEED), act))


def test_activation_spec_values(oracle):
    x = np.array(C.ACTIVATION_SPEC_VALUES, np.float32)
    for act, big in (("gelu", 15.0), ("silu", 19.0)):
        y = oracle.activation_gelu_silu(x, act)
        assert_pinned("activation_gelu_silu", f"spec_values_{act}", y)
        assert abs(y[4]) <= 1e-5 and y[8] > big  # test_activation_gelu_silu.cpp:28-44


@pytest.mark.parametrize("case", C.REDUCE_CASES, ids=lambda c: "B{}_M{}_K{}".format(*c))
def test_reduce_sum_pinned(oracle, case):
    B, M, K = case
    x = oracle.uniform(B * M * K, C.SEED).reshape(B * M, K)
    assert_pinned("reduce_sum_lastdim", f"{B}_{M}_{K}", oracle.reduce_sum_lastdim(x))


def test_reduce_sum_known_answers(oracle):
    """test_reduce_sum_lastdim.cpp:20-90, 175-187."""
    assert oracle.reduce_sum_lastdim(np.array([[1, 2, 3], [4, 5, 6]], np.float32)).tolist() == [6.0, 15.0]
    assert oracle.reduce_sum_lastdim(np.array([[1, 2, 3, 4], [5, 6, 7, 8]], np.float32)).tolist() == [10.0, 26.0]
    x = np.array([[42.0], [-17.5], [0.0], [3.14]], np.float32)
    assert np.array_equal(oracle.reduce_sum_lastdim(x), x[:, 0])
    big = oracle.reduce_sum_lastdim(np.ones((1, 100000), np.float32))
    assert_pinned("reduce_sum_lastdim", "ones_100000", big)
    assert abs(big[0] - 100000.0) <= 1.0


@pytest.mark.parametrize("case", C.TRANSPOSE_2D_CASES, ids=lambda c: "{}x{}".format(*c))
def test_transpose_2d_pinned(oracle, case):
    M, N = case
    assert_pinned("transpose_2d_4d", f"2d_f32_{M}_{N}", oracle.transpose(oracle.uniform(M * N, C.SEED).reshape(M, N), 0))
    xi = np.arange(M * N, dtype=np.int32).reshape(M, N) * np.int32(7) - np.int32(3)
    assert_pinned("transpose_2d_4d", f"2d_i32_{M}_{N}", oracle.transpose(xi, 0))


@pytest.mark.parametrize("case", C.TRANSPOSE_4D_CASES, ids=lambda c: "{}x{}x{}x{}".format(*c))
def test_transpose_4d_pinned_and_round_trip(oracle, case):
    n, c, h, w = case
    x = oracle.uniform(n * c * h * w, C.SEED).reshape(n, c, h, w)
    y = oracle.transpose(x, 1)
    assert_pinned("transpose_2d_4d", f"nchw2nhwc_{n}_{c}_{h}_{w}", y)
    assert np.array_equal(oracle.transpose(y, 2), x)  # test_transpose_2d_4d.cpp:124-126
    xh = oracle.uniform(n * c * h * w, C.SEED).reshape(n, h, w, c)
    assert_pinned("transpose_2d_4d", f"nhwc2nchw_{n}_{c}_{h}_{w}", oracle.transpose(xh, 2))


def test_codecs_round_trip_and_rne(oracle):
    import torch

    vals = np.concatenate([oracle.normal(50000, 1) * np.float32(1000), oracle.normal(50000, 2) * np.float32(1e-6),
                           np.array([0.0, -0.0, 65504.0, 65520.0, 1e-8, 6e-8, 1.00048828125], np.float32)]).astype(np.float32)
    t = torch.from_numpy(vals)
    assert np.array_equal(oracle.to_bf16(vals), t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16))
    assert np.array_equal(oracle.to_f16(vals), t.to(torch.float16).view(torch.int16).numpy().view(np.uint16))
    h = oracle.to_f16(vals)
    assert np.array_equal(oracle.from_f16(h), torch.from_numpy(h.view(np.int16)).view(torch.float16).float().numpy())
    b = oracle.to_bf16(vals)
    assert np.array_equal(oracle.from_bf16(b), torch.from_numpy(b.view(np.int16)).view(torch.bfloat16).float().numpy())


def test_live_reference_matches_oracle_when_present(oracle):
    """Where the reference goldens were compiled here (oracle/_ref), check a few fresh seeds too."""
    import oracle as omod

    if not omod.reference_available():
        pytest.skip("oracle/_ref not built")
    ref = omod.Reference()
    for seed in (1, 2, 3):
        q, k, v = C.fa_inputs(oracle, 1, 2, 70, 130, 64, 48, seed=seed)
        for causal in (0, 1):
            o, _ = oracle.flash_attention_fwd(q, k, v, 0.3, causal)
            assert np.array_equal(o, ref.flash_attention_fwd(q, k, v, 0.3, causal))
