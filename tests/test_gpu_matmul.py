"""GPU parity of matmul_bias against the pinned oracle (golden: ops/matmul_bias/golden/matmul_bias_golden.cpp).

fp32 (SIMT kernel): the reference's shape list at its tolerance 1e-4.  bf16/fp16 (tcgen05 kernel):
rel-err <= 1e-2 against the fp32 golden on the quantised inputs, including tile tails, plus the
benchmarked 8192^3 configuration checked on 128 sampled rows (both shard edges at 2/4/8 GPUs)."""
from __future__ import annotations

import numpy as np
import pytest

import cases as C
from accuracy import assert_close
from gpu_util import dev, host, quantize

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", C.MATMUL_CASES, ids=lambda c: "M{}_K{}_N{}_{}".format(c[0], c[1], c[2], "bias" if c[3] else "nobias"))
def test_matmul_f32_reference_cases(cuda, hc_lib, oracle, case):
    M, K, N, wb = case
    A, B, bias = C.matmul_inputs(oracle, M, K, N)
    out = hc_lib.matmul_bias(dev(A, "f32", oracle), dev(B, "f32", oracle), dev(bias, "f32", oracle) if wb else None)
    assert_close(oracle.matmul_bias(A, B, bias if wb else None), host(out, oracle), 1e-4, 1e-4, str(case))


def _rel_err(ref, got):
    return float(np.abs(ref - got).max() / max(np.abs(ref).max(), 1e-30))


@pytest.mark.parametrize("kind", ["bf16", "f16"])
@pytest.mark.parametrize("M,K,N", [(16, 16, 16), (64, 64, 64), (128, 128, 128), (256, 64, 16), (1, 1024, 64),
                                   (64, 32, 128), (256, 256, 64), (300, 200, 264), (129, 72, 520), (1000, 1024, 1000),
                                   # CTA-pair kernel edges: one pair tile, K of one partial block, M/N/K tails
                                   (256, 8, 256), (257, 72, 1000), (512, 8, 264), (2048, 4104, 520), (768, 64, 8)])
def test_matmul_tensor_core(cuda, hc_lib, oracle, M, K, N, kind):
    A, B, bias = C.matmul_inputs(oracle, M, K, N)
    out = hc_lib.matmul_bias(dev(A, kind, oracle), dev(B, kind, oracle), dev(bias, kind, oracle))
    path = hc_lib.load().hc_matmul_bias_last_path()
    assert path == (3 if M >= 256 else 1), f"expected the tcgen05 {'CTA-pair' if M >= 256 else 'single-CTA'} path"
    ref = oracle.matmul_bias(quantize(A, kind, oracle), quantize(B, kind, oracle), quantize(bias, kind, oracle))
    got = host(out, oracle)
    assert _rel_err(ref, got) <= 1e-2, _rel_err(ref, got)
    # elementwise: within one output rounding (2^-8 for bf16) of the fp32 golden plus accumulation-order slack
    assert_close(ref, got, 2e-2 * np.abs(ref).max() / 8, 2 ** -7 if kind == "bf16" else 2 ** -9, f"{M}x{K}x{N}")


def test_matmul_no_bias_and_identity(cuda, hc_lib, oracle):
    A = oracle.uniform(128 * 128, 7, -2, 2).reshape(128, 128)
    out = hc_lib.matmul_bias(dev(A, "bf16", oracle), dev(np.eye(128, dtype=np.float32), "bf16", oracle))
    assert np.array_equal(host(out, oracle), quantize(A, "bf16", oracle))  # exact: one product per output


def test_matmul_config_sampled_rows(cuda, hc_lib, oracle):
    """Benchmarked configuration: A, B bf16 [8192, 8192] ~ N(0,1)/sqrt(K), bias ~ N(0, 0.1); rel-err <= 1e-2 vs the
    fp32 golden on 128 sampled rows (including rows 0, 1023/1024, 2047/2048, 4095/4096, 8191)."""
    import specs

    cfg = specs.bench_config("matmul_bias")
    M, K, N = cfg["M"], cfg["K"], cfg["N"]
    sk = np.float32(1.0 / np.sqrt(K))
    A = (oracle.normal(M * K, 0) * sk).reshape(M, K)
    B = (oracle.normal(K * N, 1) * sk).reshape(K, N)
    bias = oracle.normal(N, 2, 0.0, 0.1)
    out = hc_lib.matmul_bias(dev(A, "bf16", oracle), dev(B, "bf16", oracle), dev(bias, "bf16", oracle))
    got = host(out, oracle)
    rng = np.random.default_rng(0)
    rows = np.unique(np.concatenate([[0, 1023, 1024, 2047, 2048, 4095, 4096, 6143, 6144, 8191],
                                     rng.choice(M, 118, replace=False)]))
    Aq, Bq, bq = quantize(A[rows], "bf16", oracle), quantize(B, "bf16", oracle), quantize(bias, "bf16", oracle)
    ref = oracle.matmul_bias(Aq, Bq, bq)
    assert _rel_err(ref, got[rows]) <= 1e-2
    assert np.all(np.isfinite(got))
