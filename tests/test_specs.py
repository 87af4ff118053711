"""The per-operator B200 specs (ascend-npu-harness_b200/specs/*.yaml and OPERATOR_REGISTRY.yaml, in the
schema of the harness's specs/<nn>_<op>.yaml) against everything that depends on them: the C-ABI
entry points declared in include/hc_ops.h, the tolerances the GPU tests apply, the reference suites'
own fp32 tolerances, the benchmarked configurations, and bench.py.  CPU only."""
from __future__ import annotations

import re
import sys
from pathlib import Path

import pytest

import specs

ROOT = Path(__file__).resolve().parents[1]
OPS = ["elementwise_add", "axpy_scalar_affine", "broadcast_binary", "activation_gelu_silu", "reduce_sum_lastdim",
       "transpose_2d_4d", "layer_norm", "matmul_bias", "rms_norm_rope_fused", "flash_attention_fwd_fused"]

# fp32 tolerances of the reference's own GTest suites (file:line of z-zijie/ascend-npu-harness)
REFERENCE_FP32 = {
    "flash_attention_fwd_fused": (5e-4, 5e-4),   # tests/test_flash_attention_fwd_fused.cpp:93-94
    "matmul_bias": (1e-4, 1e-4),                 # tests/test_matmul_bias.cpp:35
    "layer_norm": (1e-4, 1e-4),                  # tests/test_layer_norm.cpp:33
    "rms_norm_rope_fused": (1e-4, 1e-4),         # tests/test_rms_norm_rope_fused.cpp:37
    "activation_gelu_silu": (1e-5, 1e-5),        # tests/test_activation_gelu_silu.cpp:59
    "reduce_sum_lastdim": (1e-4, 1e-4),          # tests/test_reduce_sum_lastdim.cpp:16
    "elementwise_add": (0.0, 0.0), "axpy_scalar_affine": (0.0, 0.0), "broadcast_binary": (0.0, 0.0),
    "transpose_2d_4d": (0.0, 0.0),               # tests/test_transpose_2d_4d.cpp:41
}


def test_registry_lists_the_ten_ladder_operators():
    assert list(specs.registry()) == OPS
    for op in OPS:
        s = specs.spec(op)
        assert s["name"] == op and s["target_arch"] == "sm_100a" and s["status"] == "implemented"
        for key in ("accuracy", "performance", "benchmark", "implementation", "tests"):
            assert key in s, (op, key)
        assert s["performance"]["bound"] in ("hbm", "tensor")
        assert s["benchmark"]["warmup"] >= 3 and s["benchmark"]["iterations"] >= 5
        for f in s["tests"]["files"]:
            assert (ROOT / f).exists(), (op, f)


def test_entry_points_are_declared_in_the_c_abi():
    header = (ROOT / "include" / "hc_ops.h").read_text()
    declared = set(re.findall(r"\b(hc_\w+)\s*\(", header))
    for op in OPS:
        for ep in specs.spec(op)["implementation"]["entry_points"]:
            assert ep in declared, (op, ep)
        assert specs.registry()[op]["entry_point"] in declared


def test_kernel_names_exist_in_the_cuda_sources():
    src = "".join(p.read_text() for p in (ROOT / "ascend-npu-harness_b200" / "csrc").glob("*.cu"))
    for op in OPS:
        for k in specs.spec(op)["implementation"]["kernels"]:
            assert re.search(rf"\b{k['name']}\s*\(", src), (op, k["name"])


@pytest.mark.parametrize("op", OPS)
def test_fp32_tolerance_is_the_reference_suites(op):
    t = specs.tolerance(op, "float32")
    assert (t["abs"], t["rel"]) == REFERENCE_FP32[op]


def test_16bit_tolerances_match_the_gpu_tests():
    import test_gpu_flash_attention as fa
    import test_gpu_ops as ops

    assert fa.O_TOL_BF16 == 2e-2 and fa.LSE_TOL == 2e-3      # the benchmarked configuration's max-abs
    assert specs.tolerance("flash_attention_fwd_fused", "float16")["abs"] == 5e-3
    for op, dt, key in (("layer_norm", "bfloat16", "bf16"), ("layer_norm", "float16", "f16"),
                        ("rms_norm_rope_fused", "bfloat16", "bf16")):
        assert specs.tolerance(op, dt)["rel"] == ops.OUT_HALF_ULP[key], (op, dt)
    assert specs.tolerance("layer_norm", "bfloat16")["abs"] == 1e-2
    assert specs.tolerance("rms_norm_rope_fused", "bfloat16")["abs"] == 2e-2
    assert specs.tolerance("matmul_bias", "bfloat16")["normwise_rel"] == 1e-2
    for op in ("elementwise_add", "axpy_scalar_affine", "broadcast_binary", "transpose_2d_4d"):
        assert all(specs.tolerance(op, dt).get("bit_exact") for dt in ("bfloat16", "float16", "float32")), op


def test_backward_contract():
    """The flash-attention backward block of spec 10: entry point in the C ABI, kernels in the
    sources, tolerances equal to the GPU tests', bench configuration and FLOP ratio equal to bench.py's."""
    import test_gpu_flash_attention_bwd as bwd

    sys.path.insert(0, str(ROOT))
    import bench

    b = specs.spec("flash_attention_fwd_fused")["backward"]
    header = (ROOT / "include" / "hc_ops.h").read_text()
    for ep in b["entry_points"]:
        assert re.search(rf"\b{ep}\s*\(", header), ep
    src = "".join(p.read_text() for p in (ROOT / "ascend-npu-harness_b200" / "csrc").glob("*.cu"))
    for k in b["kernels"]:
        assert re.search(rf"\b{k['name']}\s*\(", src), k["name"]
    for dt, key in (("bfloat16", "bf16"), ("float16", "f16"), ("float32", "f32")):
        assert (b["accuracy"][dt]["normwise"], b["accuracy"][dt]["max_abs_of_max"]) == bwd.BWD_TOL[key]
    assert b["accuracy"]["bfloat16"]["normwise"] == bench.FA_BWD_TOL
    assert bench.FA_BWD_FLOP_RATIO == 2.5
    c = b["benchmark"]["config"]
    assert (c["B"], c["H"], c["S_q"], c["D"]) == (bench.FA_B, bench.FA_H, bench.FA_S, bench.FA_D)
    for f in b["tests"]["files"]:
        assert (ROOT / f).exists(), f


def test_benchmark_configurations_are_the_named_workloads():
    fa = specs.bench_config("flash_attention_fwd_fused")
    assert (fa["B"], fa["H"], fa["S_q"], fa["S_k"], fa["D"], fa["D_v"]) == (16, 32, 8192, 8192, 128, 128)
    mm = specs.bench_config("matmul_bias")
    assert (mm["M"], mm["K"], mm["N"]) == (8192, 8192, 8192)
    ln = specs.bench_config("layer_norm")
    assert (ln["rows"], ln["lastDim"], ln["eps"]) == (16384, 4096, 1e-5)
    rms = specs.bench_config("rms_norm_rope_fused")
    assert (rms["B"], rms["S"], rms["heads"], rms["H"], rms["eps"], rms["theta"]) == (8, 4096, 32, 128, 1e-6, 1e4)
    assert specs.bench_config("elementwise_add") == {"shape": [4096, 8192], "dtype": "float16"}


def test_bench_reads_the_specs():
    sys.path.insert(0, str(ROOT))
    import bench

    fa = specs.bench_config("flash_attention_fwd_fused")
    assert (bench.FA_B, bench.FA_H, bench.FA_S, bench.FA_D) == (fa["B"], fa["H"], fa["S_q"], fa["D"])
    assert bench.FA_TOL == specs.tolerance("flash_attention_fwd_fused", "bfloat16")
    assert set(bench.EXTRA_OPS) == {"flash_attention_fwd_noncausal", "flash_attention_bwd", *OPS} - \
        {"flash_attention_fwd_fused"}
