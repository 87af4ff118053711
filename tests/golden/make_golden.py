"""Generates tests/golden/reference_goldens.json from the reference harness's OWN golden functions.

The reference goldens are compiled unchanged from the reference tree by oracle/Makefile into
oracle/_ref/libref_golden.so (this script runs `make` first).  For every test case the reference
GTest suites use (tests/cases.py) it records the SHA-256 of the golden's fp32 output bytes plus a
few leading values, and the generator's own output (so the oracle's data generator is pinned too).
tests/test_oracle_pins.py recomputes each case with our oracle restatement and requires identical
bytes.  Run from the repository root:  python tests/golden/make_golden.py --ref <reference tree>
(or with HC_REFERENCE_DIR set)
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "oracle"))
sys.path.insert(0, str(ROOT / "tests"))

OUT = Path(__file__).resolve().parent / "reference_goldens.json"


def digest(a: np.ndarray) -> dict:
    a = np.ascontiguousarray(a)
    return {"sha256": hashlib.sha256(a.tobytes()).hexdigest(), "shape": list(a.shape), "dtype": str(a.dtype),
            "head": [float(v) for v in a.reshape(-1)[:6]]}


def special_fa_inputs():
    """The three hand-built FA tests (test_flash_attention_fwd_fused.cpp:183-288)."""
    out = {}
    # CausalConstraintVerification: Q = 1, K rows j>=S/2 are 100, V[j][0] = j; S=8, D=16.
    S, D = 8, 16
    q = np.ones((1, 1, S, D), np.float32)
    k = np.zeros((1, 1, S, D), np.float32)
    for j in range(S):
        k[0, 0, j, :] = 100.0 if j >= S // 2 else 1.0
    v = np.zeros((1, 1, S, D), np.float32)
    v[0, 0, :, 0] = np.arange(S, dtype=np.float32)
    out["causal_constraint"] = (q, k, v, np.float32(1.0) / np.sqrt(np.float32(D)), 1)
    # ProbabilitiesSumToOne: all-ones Q, K; V[:, 0] = 1; S=4, D=4.
    S, D = 4, 4
    v = np.zeros((1, 1, S, D), np.float32)
    v[0, 0, :, 0] = 1.0
    out["sum_to_one"] = (np.ones((1, 1, S, D), np.float32), np.ones((1, 1, S, D), np.float32), v,
                         np.float32(1.0) / np.sqrt(np.float32(D)), 0)
    return out


def generate(ref) -> dict:
    import cases as C

    g: dict = {"generator": {}, "flash_attention": {}, "flash_attention_special": {}, "matmul_bias": {},
               "layer_norm": {}, "rms_norm_rope_fused": {}, "elementwise_add": {}, "axpy_scalar_affine": {},
               "broadcast_binary": {}, "activation_gelu_silu": {}, "reduce_sum_lastdim": {}, "transpose_2d_4d": {}}
    for seed, lo, hi, n in [(C.SEED, -1.0, 1.0, 4096), (C.SEED + 1000, -1.0, 1.0, 4096), (C.SEED, -3.0, 3.0, 4096),
                            (C.SEED + 1, 0.5, 1.5, 4096), (C.SEED, -2.0, 2.0, 4096), (0, -1.0, 1.0, 4096)]:
        g["generator"][f"uniform_{seed}_{lo}_{hi}_{n}"] = digest(ref.uniform(n, seed, lo, hi))
    for S, half in [(16, 32), (128, 32), (4096, 64)]:
        c, s = ref.rope_cos_sin(S, half)
        g["generator"][f"rope_{S}_{half}"] = {"cos": digest(c), "sin": digest(s)}

    for (B, H, Sq, Sk, D, Dv, causal) in C.FA_CASES:
        q, k, v = C.fa_inputs(ref, B, H, Sq, Sk, D, Dv)
        o = ref.flash_attention_fwd(q, k, v, np.float32(C.default_scale(D)), causal)
        g["flash_attention"][f"{B}_{H}_{Sq}_{Sk}_{D}_{Dv}_{causal}"] = digest(o)
    # ScaleInvariance (test_flash_attention_fwd_fused.cpp:230-255): seeds 99/100/101, S=8, D=32, H=2.
    q = ref.uniform(2 * 8 * 32, 99).reshape(1, 2, 8, 32)
    k = ref.uniform(2 * 8 * 32, 100).reshape(1, 2, 8, 32)
    v = ref.uniform(2 * 8 * 32, 101).reshape(1, 2, 8, 32)
    base = np.float32(1.0) / np.sqrt(np.float32(32))
    g["flash_attention_special"]["scale_invariance_base"] = digest(ref.flash_attention_fwd(q, k, v, base, 0))
    g["flash_attention_special"]["scale_invariance_2k"] = digest(
        ref.flash_attention_fwd(q, (k * np.float32(2.0)).astype(np.float32), v, np.float32(base / np.float32(2.0)), 0))
    for name, (q, k, v, sc, causal) in special_fa_inputs().items():
        g["flash_attention_special"][name] = digest(ref.flash_attention_fwd(q, k, v, np.float32(sc), causal))

    for (M, K, N, wb) in C.MATMUL_CASES:
        A, Bm, bias = C.matmul_inputs(ref, M, K, N)
        g["matmul_bias"][f"{M}_{K}_{N}_{int(wb)}"] = digest(ref.matmul_bias(A, Bm, bias if wb else None))

    for (rows, dim, eps) in C.LAYER_NORM_CASES:
        x, gamma, beta = C.layer_norm_inputs(ref, rows, dim)
        g["layer_norm"][f"{rows}_{dim}_{eps}"] = digest(ref.layer_norm(x, gamma, beta, np.float32(eps)))

    for (B, S, H, rot, eps) in C.RMS_ROPE_CASES:
        x, w, cos, sin = C.rms_rope_inputs(ref, B, S, H, rot)
        g["rms_norm_rope_fused"][f"{B}_{S}_{H}_{rot}_{eps}"] = digest(
            ref.rms_norm_rope_fused(x, w, cos, sin, rot, np.float32(eps)))

    for shape in C.ELEMENTWISE_SHAPES:
        n = int(np.prod(shape))
        x, y = ref.uniform(n, C.SEED), ref.uniform(n, C.SEED + 1)
        g["elementwise_add"]["x".join(map(str, shape))] = digest(ref.elementwise_add(x, y))
    g["elementwise_add"]["hand_1234_5678"] = digest(
        ref.elementwise_add(np.array([1, 2, 3, 4], np.float32), np.array([5, 6, 7, 8], np.float32)))

    for (shape, alpha, beta) in C.AXPY_CASES:
        n = int(np.prod(shape))
        g["axpy_scalar_affine"][f"{'x'.join(map(str, shape))}_{alpha}_{beta}"] = digest(
            ref.axpy_scalar_affine(ref.uniform(n, C.SEED), alpha, beta))

    for (B, Cc, H, W, yb) in C.BROADCAST_CASES:
        x = ref.uniform(B * Cc * H * W, C.SEED).reshape(B, Cc, H, W)
        y = ref.uniform(yb * Cc, C.SEED + 1)
        bias = ref.uniform(Cc, C.SEED + 2)
        g["broadcast_binary"][f"{B}_{Cc}_{H}_{W}_{yb}"] = digest(ref.broadcast_binary(x, y, bias, yb))

    for (shape, act) in C.ACTIVATION_CASES:
        n = int(np.prod(shape))
        g["activation_gelu_silu"][f"{'x'.join(map(str, shape))}_{act}"] = digest(
            ref.activation_gelu_silu(ref.uniform(n, C.SEED), act))
    for act in ("gelu", "silu"):
        g["activation_gelu_silu"][f"spec_values_{act}"] = digest(
            ref.activation_gelu_silu(np.array(C.ACTIVATION_SPEC_VALUES, np.float32), act))

    for (B, M, K) in C.REDUCE_CASES:
        x = ref.uniform(B * M * K, C.SEED).reshape(B * M, K)
        g["reduce_sum_lastdim"][f"{B}_{M}_{K}"] = digest(ref.reduce_sum_lastdim(x))
    g["reduce_sum_lastdim"]["ones_100000"] = digest(ref.reduce_sum_lastdim(np.ones((1, 100000), np.float32)))

    for (M, N) in C.TRANSPOSE_2D_CASES:
        xf = ref.uniform(M * N, C.SEED).reshape(M, N)
        g["transpose_2d_4d"][f"2d_f32_{M}_{N}"] = digest(ref.transpose(xf, 0))
        xi = np.arange(M * N, dtype=np.int32).reshape(M, N) * np.int32(7) - np.int32(3)
        g["transpose_2d_4d"][f"2d_i32_{M}_{N}"] = digest(ref.transpose(xi, 0))
    for (n, c, h, w) in C.TRANSPOSE_4D_CASES:
        x = ref.uniform(n * c * h * w, C.SEED).reshape(n, c, h, w)
        g["transpose_2d_4d"][f"nchw2nhwc_{n}_{c}_{h}_{w}"] = digest(ref.transpose(x, 1))
        xh = ref.uniform(n * c * h * w, C.SEED).reshape(n, h, w, c)
        g["transpose_2d_4d"][f"nhwc2nchw_{n}_{c}_{h}_{w}"] = digest(ref.transpose(xh, 2))
    return g


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("HC_REFERENCE_DIR"),
                    help="path of the reference harness source tree (default: $HC_REFERENCE_DIR)")
    a = ap.parse_args()
    import oracle

    oracle.build(a.ref)
    ref = oracle.Reference()
    g = generate(ref)
    g["_about"] = ("SHA-256 of fp32 outputs of the reference harness's own golden functions "
                   "(compiled from its sources by oracle/Makefile) on the inputs of its GTest suites; "
                   "generated by tests/golden/make_golden.py")
    OUT.write_text(json.dumps(g, indent=1, sort_keys=True) + "\n")
    n = sum(len(v) for k, v in g.items() if isinstance(v, dict))
    print(f"wrote {OUT} ({n} entries)")


if __name__ == "__main__":
    main()
