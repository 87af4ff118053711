"""Accuracy comparison with the reference harness's semantics.

compare() restates harness::accuracy::CompareArrays (include/harness/accuracy.hpp:62-125): an
element fails only if |e-a| > abs_tol AND rel > rel_tol, rel taken against |expected| (or
|actual| when expected is ~0).  Unlike the reference it also reports max-abs / max-rel over ALL
elements (the reference tracks them over failing elements only, accuracy.hpp:88-95)."""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass
class Report:
    passed: bool
    n: int
    mismatches: int
    max_abs: float
    max_rel: float
    first_bad: list

    def __str__(self) -> str:
        return (f"passed={self.passed} n={self.n} mismatches={self.mismatches} max_abs={self.max_abs:.3e} "
                f"max_rel={self.max_rel:.3e} first={self.first_bad[:4]}")


def compare(expected, actual, abs_tol: float, rel_tol: float) -> Report:
    e = np.asarray(expected, np.float64).reshape(-1)
    a = np.asarray(actual, np.float64).reshape(-1)
    assert e.shape == a.shape, (e.shape, a.shape)
    err = np.abs(e - a)
    denom = np.where(np.abs(e) > 1e-12, np.abs(e), np.where(np.abs(a) > 1e-12, np.abs(a), np.inf))
    rel = np.where(np.isfinite(denom), err / denom, 0.0)
    bad = (err > abs_tol) & (rel > rel_tol)
    bad |= ~np.isfinite(a) & np.isfinite(e)
    idx = np.flatnonzero(bad)
    return Report(passed=idx.size == 0, n=e.size, mismatches=int(idx.size),
                  max_abs=float(err.max()) if err.size else 0.0,
                  max_rel=float(rel.max()) if rel.size else 0.0,
                  first_bad=[(int(i), float(e[i]), float(a[i])) for i in idx[:8]])


def assert_close(expected, actual, abs_tol: float, rel_tol: float, what: str = "") -> Report:
    r = compare(expected, actual, abs_tol, rel_tol)
    assert r.passed, f"{what}: {r}"
    return r
