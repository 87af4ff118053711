"""Per-operator B200 contracts (specs/*.yaml, OPERATOR_REGISTRY.yaml in this package).

The specs keep the harness's spec schema (specs/<nn>_<op>.yaml and OPERATOR_REGISTRY.yaml of
z-zijie/ascend-npu-harness) and record, per operator: element types, the kernels and when each is
taken, the accuracy tolerances the GPU tests apply, the roofline bound, and the benchmark
configuration.  bench.py reads its configurations and accuracy tolerances through this module.
"""
from __future__ import annotations

from functools import lru_cache
from pathlib import Path

import yaml

HERE = Path(__file__).resolve().parent
REGISTRY = HERE / "OPERATOR_REGISTRY.yaml"


@lru_cache(maxsize=None)
def registry() -> dict:
    """The registry's `operators` mapping: op name -> entry (spec path relative to this package)."""
    return yaml.safe_load(REGISTRY.read_text())["operators"]


@lru_cache(maxsize=None)
def spec(op: str) -> dict:
    """The parsed spec of one ladder operator."""
    entry = registry().get(op)
    if entry is None:
        raise KeyError(f"{op!r} is not in {REGISTRY.name}")
    return yaml.safe_load((HERE / entry["spec"]).read_text())


def bench_config(op: str) -> dict:
    """The benchmark configuration (shapes, element type, op parameters) of `op`."""
    return dict(spec(op)["benchmark"]["config"])


def tolerance(op: str, dtype: str) -> dict:
    """Accuracy tolerances of `op` for an element type name ('bfloat16', 'float16', 'float32')."""
    return dict(spec(op)["accuracy"][dtype])
