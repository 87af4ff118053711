"""The reference harness's OWN GoogleTest suites (tests/test_<op>.cpp) and benches
(ops/<op>/bench/bench_<op>.cpp), compiled unchanged against the B200 runner seam by
tests/cpp/reference_suite.mk (built from the reference tree by __graft_entry__.build(); the binaries
travel to the GPU machine, the reference tree does not).

  * CPU: every binary lists the reference's test count, and the harness-core suite passes (its
    device-availability test reports "no device" here instead of crashing).
  * GPU: every suite passes with each runner entry point executing on the B200 (no golden
    fallback exists on that path), and the benches time the GPU runners through the reference's
    own timing loop.

The expected counts are the reference suites' own: TEST/TEST_F bodies plus one test per
INSTANTIATE_TEST_SUITE_P value."""
from __future__ import annotations

import re
import subprocess
from pathlib import Path

import pytest

BIN = Path(__file__).resolve().parent / "cpp" / "_bin" / "reference"
SUITES = {"harness_core": 13, "elementwise_add": 11, "axpy_scalar_affine": 20, "broadcast_binary": 13,
          "activation_gelu_silu": 8, "reduce_sum_lastdim": 25, "transpose_2d_4d": 21, "layer_norm": 15,
          "rms_norm_rope_fused": 6, "matmul_bias": 18, "flash_attention_fwd_fused": 17}
BENCHES = {"flash_attention_fwd_fused": ["1", "2", "1024", "1024", "128"], "layer_norm": [], "elementwise_add": []}


def _binary(name: str) -> Path:
    p = BIN / name
    if not p.exists():
        pytest.skip(f"{p.name} not built (make -f tests/cpp/reference_suite.mk REF=<reference tree>)")
    return p


def _run(args, timeout=600) -> subprocess.CompletedProcess:
    return subprocess.run([str(a) for a in args], capture_output=True, text=True, timeout=timeout)


@pytest.mark.parametrize("op", sorted(SUITES))
def test_reference_suite_lists_its_tests(op):
    r = _run([_binary(f"test_{op}"), "--gtest_list_tests"], 60)
    assert r.returncode == 0, r.stderr
    assert len(r.stdout.split()) == SUITES[op], r.stdout


def test_reference_harness_core_suite_on_cpu():
    r = _run([_binary("test_harness_core")], 120)
    assert r.returncode == 0, r.stdout[-4000:]
    assert f"[  PASSED  ] {SUITES['harness_core']} tests." in r.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("op", sorted(SUITES))
def test_reference_suite_on_gpu(cuda, op):
    r = _run([_binary(f"test_{op}")], 1200)
    assert r.returncode == 0, r.stdout[-8000:] + r.stderr[-2000:]
    m = re.search(r"\[  PASSED  \] (\d+) tests\.", r.stdout)
    skipped = re.search(r"\[  SKIPPED \] (\d+) tests\.", r.stdout)
    assert m and int(m.group(1)) + (int(skipped.group(1)) if skipped else 0) == SUITES[op], r.stdout[-3000:]
    assert "FAILED" not in r.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("op", sorted(BENCHES))
def test_reference_bench_on_gpu(cuda, op):
    r = _run([_binary(f"bench_{op}"), *BENCHES[op]], 600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    print(r.stdout.strip())
    assert re.search(r"\d", r.stdout)
