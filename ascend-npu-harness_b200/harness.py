"""Command-line driver of the B200 operator ladder, the counterpart of the harness's
scripts/harness.py (build / test / bench / status, scripts/harness.py:238-299, 329-352) with a
`cuda` mode in place of the `npu` one:

  python ascend-npu-harness_b200/harness.py build  --mode host|cuda
  python ascend-npu-harness_b200/harness.py test   --mode host|cuda [--op <op>]
  python ascend-npu-harness_b200/harness.py bench  <op> [--gpus N]
  python ascend-npu-harness_b200/harness.py status

  build --mode host   the CPU checkers (oracle/) and the C++ host-layer tests
  build --mode cuda   libhc_b200.so (nvcc, sm_100a), libhc_harness.so, libhc_torch.so, and the
                      reference's own suites against the B200 runner seam when HC_REFERENCE_DIR
                      names the reference tree
  test  --mode host   pytest -m "not gpu" (CPU); with --op, that operator's oracle pins and the
                      listing of the reference's own suite for it
  test  --mode cuda   pytest -m gpu (a B200); with --op, the spec's test files filtered to the op,
                      plus the reference's own suite for it when built
  bench <op>          bench.py for that operator's benchmark configuration (the headline for
                      flash_attention_fwd_fused), one JSON line
  status              the operator registry (OPERATOR_REGISTRY.yaml) with each spec's bound and
                      benchmark configuration

Every command records its command line, exit status and output tail as JSON under
.harness_runs/<timestamp>_<command>/ at the repository root (as the reference keeps
.npu-harness/runs/), and exits with the status of what it ran.  --dry-run prints the commands only.
"""
from __future__ import annotations

import argparse
import json
import os
import shlex
import subprocess
import sys
import time
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
sys.path.insert(0, str(HERE))

import specs  # noqa: E402

RUNS = ROOT / ".harness_runs"


def _record(name: str, results: list[dict]) -> Path:
    run_dir = RUNS / f"{time.strftime('%Y%m%d_%H%M%S')}_{name}"
    run_dir.mkdir(parents=True, exist_ok=True)
    (run_dir / "result.json").write_text(json.dumps(results, indent=1) + "\n")
    return run_dir


def _run(cmds: list[list[str]], name: str, dry: bool, env: dict | None = None) -> int:
    """Runs the commands in order (stopping at the first failure) and records them."""
    if dry:
        for c in cmds:
            print(shlex.join(c))
        return 0
    results, rc = [], 0
    for c in cmds:
        print(f"=== {shlex.join(c)}", flush=True)
        t0 = time.time()
        p = subprocess.run(c, cwd=ROOT, env={**os.environ, **(env or {})}, capture_output=True, text=True)
        out = p.stdout + p.stderr
        print(out[-3000:], flush=True)
        results.append({"cmd": shlex.join(c), "rc": p.returncode, "seconds": round(time.time() - t0, 1),
                        "tail": out[-4000:]})
        rc = p.returncode
        if rc:
            break
    run_dir = _record(name, results)
    print(f"{name}: {'PASSED' if rc == 0 else f'FAILED (exit code {rc})'}; run dir {run_dir}")
    return rc


def _op_names() -> list[str]:
    return list(specs.registry())


def cmd_build(a) -> int:
    py = sys.executable
    if a.mode == "host":
        cmds = [["make", "-s", "-C", "oracle"], ["make", "-s", "-C", "tests/cpp"]]
    else:
        cmds = [[py, str(HERE / "build.py")],
                [py, "-c", f"import sys; sys.path.insert(0, {str(HERE)!r}); import build; build.build_host(); "
                           "build.build_torch()"]]
        ref = os.environ.get("HC_REFERENCE_DIR")
        if ref:
            cmds.append(["make", "-s", "-j8", "-f", "tests/cpp/reference_suite.mk", f"REF={ref}"])
    return _run(cmds, f"build_{a.mode}", a.dry_run)


def _op_filter(op: str, mode: str) -> list[str]:
    """pytest arguments selecting one operator.  cuda: its spec's GPU test files (filtered by name
    where a file covers several operators); host: the oracle's pins against the reference goldens
    and the reference suite's build for that operator."""
    if mode == "host":
        return ["tests/test_oracle_pins.py", "tests/test_reference_suites.py", "-k", op]
    files = [f for f in specs.spec(op)["tests"]["files"] if f.endswith(".py")]
    shared = any(f.endswith("test_gpu_ops.py") for f in files)
    return files + (["-k", op] if shared else [])


def cmd_test(a) -> int:
    py = sys.executable
    marker = "gpu" if a.mode == "cuda" else "not gpu"
    if a.op:
        if a.op not in specs.registry():
            print(f"unknown operator {a.op!r}; one of: {', '.join(_op_names())}")
            return 2
        cmds = [[py, "-m", "pytest", "-q", "-m", marker, *_op_filter(a.op, a.mode)]]
        suite = ROOT / "tests" / "cpp" / "_bin" / "reference" / f"test_{a.op}"
        if a.mode == "cuda" and suite.exists():
            cmds.append([str(suite)])
    else:
        cmds = [[py, "-m", "pytest", "-q", "-m", marker, "tests"]]
    return _run(cmds, f"test_{a.mode}" + (f"_{a.op}" if a.op else ""), a.dry_run)


def cmd_bench(a) -> int:
    if a.op_name not in specs.registry():
        print(f"unknown operator {a.op_name!r}; one of: {', '.join(_op_names())}")
        return 2
    bench = [str(ROOT / "bench.py"), "--gpus", str(a.gpus)]
    if a.op_name == "flash_attention_fwd_fused":
        args = bench + ["--no-extras"]
    else:
        args = bench + ["--only", a.op_name]
    if a.gpus > 1:
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={a.gpus}",
               "--master-addr", "127.0.0.1", "--master-port", str(a.port), *args]
    else:
        cmd = [sys.executable, *args]
    return _run([cmd], f"bench_{a.op_name}", a.dry_run)


def cmd_status(a) -> int:
    for op, entry in specs.registry().items():
        s = specs.spec(op)
        flags = ", ".join(f"{k}={entry[k]}" for k in ("built_device", "tested_device", "accuracy") if k in entry)
        print(f"{op:28s} {s['performance']['bound']:6s} {flags}  bench {s['benchmark']['config']}")
    return 0


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="command", required=True)
    p = sub.add_parser("build")
    p.add_argument("--mode", choices=["host", "cuda"], default="host")
    p.add_argument("--dry-run", action="store_true")
    p = sub.add_parser("test")
    p.add_argument("--mode", choices=["host", "cuda"], default="host")
    p.add_argument("--op", help="operator name (OPERATOR_REGISTRY.yaml)")
    p.add_argument("--dry-run", action="store_true")
    p = sub.add_parser("bench")
    p.add_argument("op_name")
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--port", type=int, default=29531)
    p.add_argument("--dry-run", action="store_true")
    sub.add_parser("status")
    a = ap.parse_args(argv)
    return {"build": cmd_build, "test": cmd_test, "bench": cmd_bench, "status": cmd_status}[a.command](a)


if __name__ == "__main__":
    sys.exit(main())
