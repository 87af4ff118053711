"""The FMA-pipe exponential of the flash-attention softmax (exp2_poly2 in exp2_poly.cuh):
its constants are the Remez minimax fit that tests/exp2_poly_fit.py derives, and the exact fp32
device sequence (emulated here) stays within 1e-4 relative error of 2^x on the range the kernel
uses it for.  CPU only."""
from __future__ import annotations

import re
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(Path(__file__).resolve().parent))

import exp2_poly_fit as fit  # noqa: E402


def kernel_constants():
    src = (ROOT / "ascend-npu-harness_b200" / "csrc" / "exp2_poly.cuh").read_text()
    return [float(re.search(rf"kExp2C{i} = ([0-9.eE+-]+)f;", src).group(1)) for i in range(4)]


def test_constants_are_the_remez_fit():
    c, err = fit.remez_exp2()
    assert err < 8e-5
    np.testing.assert_allclose(kernel_constants(), c, rtol=0, atol=2e-7)


def test_device_sequence_accuracy():
    c = kernel_constants()
    x = np.concatenate([np.linspace(-30.0, 8.5, 400001, dtype=np.float32),
                        np.array([-0.5, 0.5, -1.5, 1.5, 0.0, 8.0, -119.0], np.float32)])
    got = fit.emulate_exp2_poly(x, c).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    assert np.max(np.abs(got - ref) / ref) < 1e-4
    # far below the clamp the result is a tiny positive normal, never garbage
    tiny = fit.emulate_exp2_poly(np.array([-1e4, -200.0, -121.0], np.float32), c)
    assert np.all(tiny > 0) and np.all(tiny < 1e-35)
