"""Derives the cubic used by exp2_poly2() in ops_attention.cu: the minimax-relative-error
polynomial p(f) ~ 2^f on [-1/2, 1/2], computed with the Remez exchange algorithm.

The flash-attention softmax evaluates 2^x either on the MUFU unit (ex2.approx) or, for 1/4 of the
keys of unmasked tiles at head dim 64, on the FMA pipe as 2^x = 2^n * p(f) with n = rint(x),
f = x - n.  Running this script prints
the four fp32 coefficients and the achieved maximum relative error (about 7.5e-5, well below the
2^-9 relative precision of the bf16 probabilities the kernel feeds to the tensor core).
"""
from __future__ import annotations

import numpy as np


def remez_exp2(degree: int = 3, lo: float = -0.5, hi: float = 0.5, iterations: int = 40):
    """Minimax fit of 2^f with relative-error weight; returns (coefficients c0..cd, max rel err)."""
    n = degree + 2
    # Chebyshev extrema as the initial reference set.
    x = 0.5 * (lo + hi) + 0.5 * (hi - lo) * np.cos(np.pi * np.arange(n)[::-1] / (n - 1))
    grid = np.linspace(lo, hi, 200001)
    coeffs = None
    for _ in range(iterations):
        # Solve p(x_i) - 2^{x_i} = (-1)^i E 2^{x_i} for the coefficients and the level E.
        A = np.zeros((n, n))
        for i in range(n):
            A[i, : degree + 1] = x[i] ** np.arange(degree + 1)
            A[i, degree + 1] = (-1) ** i * 2.0 ** x[i]
        sol = np.linalg.solve(A, 2.0 ** x)
        coeffs = sol[: degree + 1]
        err = (np.polyval(coeffs[::-1], grid) - 2.0 ** grid) / 2.0 ** grid
        # New reference set: the extremum of |err| in each interval of constant sign.
        segments = np.split(np.arange(grid.size), np.where(np.diff(np.sign(err)) != 0)[0] + 1)
        extrema = [seg[np.argmax(np.abs(err[seg]))] for seg in segments]
        if len(extrema) != n:
            break
        x = grid[extrema]
    err = (np.polyval(coeffs[::-1], grid) - 2.0 ** grid) / 2.0 ** grid
    return coeffs, float(np.abs(err).max())


def emulate_exp2_poly(x: np.ndarray, coeffs) -> np.ndarray:
    """fp32 emulation of the device sequence (clamp, 1.5*2^23 rounding, Horner, exponent add)."""
    c = [np.float32(v) for v in coeffs]
    x = np.maximum(np.asarray(x, np.float32), np.float32(-120.0))
    magic = np.float32(12582912.0)
    t = (x + magic).astype(np.float32)
    f = (x - (t - magic).astype(np.float32)).astype(np.float32)
    p = (c[3] * f + c[2]).astype(np.float32)
    p = (p * f + c[1]).astype(np.float32)
    p = (p * f + c[0]).astype(np.float32)
    n = (t.view(np.int32) << 23).astype(np.int32)
    return (p.view(np.int32) + n).astype(np.int32).view(np.float32)


if __name__ == "__main__":
    c, e = remez_exp2()
    print("c0..c3 =", ", ".join(f"{np.float32(v)!r}" for v in c), f"  max relative error {e:.3e}")
