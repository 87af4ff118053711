"""Test cases of the reference harness's own GTest suites, restated as data.

Each list mirrors one reference test file (shapes, seeds, value ranges and scalars), so the
golden fixtures (tests/golden/make_golden.py), the oracle pins and the GPU parity tests all
exercise the same inputs the reference tests use.  Inputs come from the harness generator
(mt19937_64 + uniform_real_distribution<float>, include/harness/test_utils.hpp:39-46), which the
oracle reproduces bit for bit.
"""
from __future__ import annotations

SEED = 20260522  # include/harness/test_utils.hpp:20

# tests/test_flash_attention_fwd_fused.cpp:121-178  (B, H, S_q, S_k, D, D_v, causal)
FA_CASES = [
    (1, 4, 1, 1, 32, 32, 0),
    (1, 1, 16, 16, 64, 64, 0),
    (1, 8, 16, 16, 32, 32, 0),
    (2, 4, 16, 16, 64, 64, 0),
    (1, 4, 8, 8, 32, 32, 1),
    (1, 1, 16, 16, 64, 64, 1),
    (2, 4, 32, 32, 128, 128, 1),
    (1, 4, 8, 16, 64, 64, 0),
    (1, 2, 4, 32, 128, 128, 0),
    (1, 4, 64, 64, 64, 64, 0),
    (1, 4, 64, 64, 64, 64, 1),
    (1, 2, 128, 128, 32, 32, 0),
    (1, 4, 8, 8, 64, 32, 0),
    (1, 4, 16, 16, 128, 64, 1),
]


def fa_inputs(oracle, B, H, S_q, S_k, D, D_v, seed=SEED):
    """test_flash_attention_fwd_fused.cpp:74-79: U[-1,1] with seeds seed, seed+1000, seed+2000."""
    q = oracle.uniform(B * H * S_q * D, seed).reshape(B, H, S_q, D)
    k = oracle.uniform(B * H * S_k * D, seed + 1000).reshape(B, H, S_k, D)
    v = oracle.uniform(B * H * S_k * D_v, seed + 2000).reshape(B, H, S_k, D_v)
    return q, k, v


# tests/test_matmul_bias.cpp:43-67  (M, K, N, with_bias)
MATMUL_CASES = [
    (1, 1, 1, False), (16, 16, 16, False), (64, 64, 64, False), (128, 128, 128, False), (256, 64, 16, False),
    (1, 1024, 64, False), (1, 1, 1, True), (16, 16, 16, True), (64, 32, 128, True), (128, 128, 128, True),
    (256, 256, 64, True), (1, 1024, 64, True), (64, 64, 1, False), (1, 1, 64, False), (1, 1024, 1, True),
]


def matmul_inputs(oracle, M, K, N, seed=SEED):
    """test_matmul_bias.cpp:22-25: A, B ~ U[-2,2], bias ~ U[-0.5,0.5]."""
    A = oracle.uniform(M * K, seed, -2.0, 2.0).reshape(M, K)
    B = oracle.uniform(K * N, seed + 1, -2.0, 2.0).reshape(K, N)
    bias = oracle.uniform(N, seed + 2, -0.5, 0.5)
    return A, B, bias


# tests/test_layer_norm.cpp:40-56  (rows, last_dim, eps)
LAYER_NORM_CASES = [
    (1, 16, 1e-5), (3, 64, 1e-5), (1, 128, 1e-5), (64, 768, 1e-5), (4, 1024, 1e-5), (1, 4096, 1e-5), (257, 64, 1e-5),
    (1, 64, 1e-5), (16, 768, 1e-5), (32, 256, 1e-5), (512, 128, 1e-5), (64, 768, 1e-6),
]


def layer_norm_inputs(oracle, rows, dim, seed=SEED):
    """test_layer_norm.cpp:19-23: x ~ U[-3,3], gamma ~ U[0.5,1.5], beta ~ U[-0.5,0.5]."""
    x = oracle.uniform(rows * dim, seed, -3.0, 3.0).reshape(rows, dim)
    gamma = oracle.uniform(dim, seed + 1, 0.5, 1.5)
    beta = oracle.uniform(dim, seed + 2, -0.5, 0.5)
    return x, gamma, beta


# tests/test_rms_norm_rope_fused.cpp:43-48  (B, S, H, rotary_dim, eps)
RMS_ROPE_CASES = [
    (1, 1, 64, 32, 1e-5), (1, 16, 128, 64, 1e-5), (2, 16, 256, 128, 1e-5), (4, 128, 128, 64, 1e-5),
    (1, 16, 128, 64, 1e-6), (1, 16, 64, 64, 1e-5),
]


def rms_rope_inputs(oracle, B, S, H, rot, seed=SEED):
    """test_rms_norm_rope_fused.cpp:19-24: x, weight ~ U[-1,1]; cos/sin from generate_rope_cos_sin."""
    x = oracle.uniform(B * S * H, seed).reshape(B, S, H)
    w = oracle.uniform(H, seed + 1)
    cos, sin = oracle.rope_cos_sin(S, rot // 2)
    return x, w, cos, sin


# tests/test_elementwise_add.cpp:81-89 shapes
ELEMENTWISE_SHAPES = [(1,), (8,), (1024,), (3, 7), (4, 16, 64), (2, 3, 32, 128)]

# tests/test_axpy_scalar_affine.cpp:93-111  (shape, alpha, beta)
AXPY_CASES = [
    ((1,), 0.0, 0.0), ((1,), 1.0, 1.0), ((1,), -1.0, -1.0), ((1,), 0.5, 0.5), ((1,), -2.25, -2.25),
    ((17,), 0.0, 1.0), ((17,), 1.0, 0.0), ((17,), -1.0, 0.5), ((1024,), 0.5, -1.0), ((1024,), -2.25, 1.0),
    ((4097,), 0.5, 0.0), ((4097,), -2.25, -2.25), ((32, 128), 0.0, 0.0), ((32, 128), 1.0, -1.0),
    ((32, 128), -2.25, 0.5),
]

# tests/test_broadcast_binary.cpp:116-128  (B, C, H, W, y_batch)
BROADCAST_CASES = [
    (1, 1, 1, 1, 1), (1, 3, 7, 7, 1), (2, 16, 32, 32, 1), (4, 64, 63, 63, 1), (1, 3, 32, 64, 1), (2, 1, 32, 32, 2),
    (1, 1, 63, 63, 1), (4, 16, 1, 1, 1), (1, 64, 7, 7, 1),
]

# tests/test_activation_gelu_silu.cpp:64-69  (shape, act)
ACTIVATION_CASES = [((128,), "gelu"), ((1024,), "gelu"), ((8, 512), "silu"), ((2, 16, 128), "silu")]
ACTIVATION_SPEC_VALUES = [-20.0, -10.0, -5.0, -1.0, 0.0, 1.0, 5.0, 10.0, 20.0]  # :28-44

# tests/test_reduce_sum_lastdim.cpp:114-165  (B, M, K)
REDUCE_CASES = [
    (1, 1, 1), (1, 1, 7), (1, 1, 32), (1, 1, 128), (1, 1, 1024), (1, 1, 4096), (1, 3, 128), (1, 64, 32),
    (1, 64, 4096), (1, 257, 7), (1, 1, 32), (2, 3, 128), (8, 64, 1024), (1, 64, 1), (2, 1, 4096), (8, 1, 7),
]

# tests/test_transpose_2d_4d.cpp:48-126
TRANSPOSE_2D_CASES = [(1, 1), (3, 7), (32, 32), (128, 64), (257, 129)]
TRANSPOSE_4D_CASES = [(1, 3, 224, 224), (2, 16, 32, 32), (4, 7, 13, 17)]


def default_scale(D: int) -> float:
    """1.0f / std::sqrt(float(D)) in fp32 arithmetic (test_flash_attention_fwd_fused.cpp:72)."""
    import numpy as np

    return float(np.float32(1.0) / np.sqrt(np.float32(D)))
