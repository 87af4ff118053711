"""The command-line driver (ascend-npu-harness_b200/harness.py, the counterpart of the harness's
scripts/harness.py build/test/bench/status with a cuda mode): the registry listing, the commands each
mode runs, a host-mode operator run on CPU, and (-m gpu) a cuda-mode operator test and a bench run."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
CLI = ROOT / "ascend-npu-harness_b200" / "harness.py"


def cli(*args, timeout=600) -> subprocess.CompletedProcess:
    return subprocess.run([sys.executable, str(CLI), *args], cwd=ROOT, capture_output=True, text=True,
                          timeout=timeout)


def test_status_lists_every_operator():
    r = cli("status")
    assert r.returncode == 0, r.stderr
    names = [line.split()[0] for line in r.stdout.splitlines()]
    assert names == ["elementwise_add", "axpy_scalar_affine", "broadcast_binary", "activation_gelu_silu",
                     "reduce_sum_lastdim", "transpose_2d_4d", "layer_norm", "matmul_bias", "rms_norm_rope_fused",
                     "flash_attention_fwd_fused"]


def test_modes_run_the_expected_commands():
    r = cli("test", "--mode", "cuda", "--op", "layer_norm", "--dry-run")
    assert r.returncode == 0
    assert "-m gpu tests/test_gpu_ops.py -k layer_norm" in r.stdout
    r = cli("test", "--mode", "host", "--dry-run")
    assert "-m 'not gpu' tests" in r.stdout
    r = cli("bench", "matmul_bias", "--gpus", "2", "--dry-run")
    assert "torch.distributed.run" in r.stdout and "--nproc-per-node=2" in r.stdout and "--only matmul_bias" in r.stdout
    r = cli("build", "--mode", "cuda", "--dry-run")
    assert "build.py" in r.stdout
    assert cli("test", "--op", "no_such_op").returncode == 2


def _last_run(name: str) -> dict:
    runs = sorted((ROOT / ".harness_runs").glob(f"*_{name}"))
    assert runs, name
    return json.loads((runs[-1] / "result.json").read_text())


def test_host_mode_operator_run():
    r = cli("test", "--mode", "host", "--op", "elementwise_add")
    assert r.returncode == 0, r.stdout[-3000:]
    assert "PASSED" in r.stdout
    assert _last_run("test_host_elementwise_add")[0]["rc"] == 0


@pytest.mark.gpu
def test_cuda_mode_operator_run(cuda):
    r = cli("test", "--mode", "cuda", "--op", "elementwise_add", timeout=1200)
    assert r.returncode == 0, r.stdout[-4000:]
    res = _last_run("test_cuda_elementwise_add")
    assert [x["rc"] for x in res] == [0, 0]  # the pytest GPU tests, then the reference's own suite


@pytest.mark.gpu
def test_bench_through_the_cli(cuda):
    r = cli("bench", "elementwise_add", timeout=600)
    assert r.returncode == 0, r.stdout[-3000:]
    line = [x for x in r.stdout.splitlines() if x.startswith("{")][-1]
    entry = json.loads(line)
    assert entry["only"] == "elementwise_add" and entry["pass"] and entry["unit"] == "GB/s"
