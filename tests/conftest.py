"""pytest configuration: the `gpu` marker, import paths and shared fixtures.

Tests marked `gpu` need a CUDA device (B200); everything else runs on CPU.  The product library
is loaded from ascend-npu-harness_b200/lib (built by __graft_entry__.build()); the oracle from
oracle/ (built on demand by its Makefile).
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "ascend-npu-harness_b200"
for p in (PKG, ROOT / "oracle", ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


@pytest.fixture(scope="session")
def oracle():
    import oracle as o

    return o.Oracle()


@pytest.fixture(scope="session")
def hc_lib():
    """The product library; built first if missing (nvcc cross-compiles without a GPU)."""
    import hc

    if not hc.LIB_PATH.exists():
        sys.path.insert(0, str(PKG))
        import build

        build.build()
    return hc


@pytest.fixture(scope="session")
def cuda(hc_lib):
    """A CUDA device for gpu-marked tests: fails loudly (never skips) when there is none."""
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu test collected on a machine without CUDA (run with -m 'not gpu' here)")
    torch.cuda.init()
    return torch.device("cuda:0")
