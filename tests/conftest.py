"""Shared pytest setup.

* ``gpu`` marks tests that need a B200 (they call the CUDA path through the
  C-ABI).  Without a GPU they are skipped; the CPU suite runs with
  ``-m "not gpu"``.
* The drop-in package lives in ``fp-emulation_b200/`` (the counterpart of the
  reference's ``src/``), and the oracle in ``oracle/``; both go on sys.path.
"""
from __future__ import annotations

import math
import sys
from fractions import Fraction
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
for p in (REPO / "fp-emulation_b200", REPO):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); calls the CUDA path")


def _has_gpu() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA GPU in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def golden_names():
    return sorted(p.stem for p in GOLDEN.glob("*.npz")
                  if not p.stem.startswith("ref_convert") and not p.stem.startswith("ref_backward"))


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def exact_fma(a: float, b: float, c: float) -> float:
    """fma(a, b, c) with one rounding (Python 3.12 has no math.fma)."""
    if not all(map(math.isfinite, (a, b, c))):
        return a * b + c
    return float(Fraction(a) * Fraction(b) + Fraction(c))


def compensated_matmul(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    """TwoProduct + compensated summation, the reference's ground truth for tiny
    sizes (reference tests/conftest.py:18-41), with an exact-fma shim."""
    p, q = A.shape
    r = B.shape[1]
    C = np.zeros((p, r))
    for i in range(p):
        for j in range(r):
            s, e = 0.0, 0.0
            for k in range(q):
                a, b = float(A[i, k]), float(B[k, j])
                prod = a * b
                ep = exact_fma(a, b, -prod)
                y = prod - e
                t = s + y
                e = (t - s) - y
                s = t
                s += ep
            C[i, j] = s
    return C


def ulp_diff(x: np.ndarray, y: np.ndarray) -> np.ndarray:
    """|x - y| in units of y's ulp (0 where both are equal, inf for NaN mismatch)."""
    x = np.asarray(x, dtype=np.float64)
    y = np.asarray(y, dtype=np.float64)
    same = (x == y) | (np.isnan(x) & np.isnan(y))
    u = np.spacing(np.abs(y))
    d = np.abs(x - y) / np.where(u > 0, u, np.finfo(np.float64).tiny)
    return np.where(same, 0.0, d)
