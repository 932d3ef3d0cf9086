"""Config 2's modulus sweep: accuracy against n_mod.

The GPU product equals the oracle bit for bit at every modulus count
(``test_gpu_parity.py::test_modulus_sweep``), so the oracle's accuracy here is
the GPU's.  Inputs: (U(0,1) - 0.5) * exp(phi * N(0,1)), n = 384, phi in
{0.5, 1, 2}.  Reference: the compensated dot product Dot2 (Ogita, Rump and
Oishi 2005: TwoProduct by Dekker's split, TwoSum), whose own error is about
k eps^2 |A||B|, far below what is measured.  Error per entry is reported in
units of eps * (|A||B|)_ij; the reference default n_mod (24 at k = 384) must be
within the split-aware bound the reference itself satisfies.  Run with ``-s``
to print the table.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import ozaki_oracle as oo

EPS = 2.0 ** -53


def _two_sum(a, b):
    s = a + b
    v = s - a
    return s, (a - (s - v)) + (b - v)


def _split(a):
    c = 134217729.0 * a  # 2^27 + 1
    hi = c - (c - a)
    return hi, a - hi


def _two_prod(a, b):
    p = a * b
    ah, al = _split(a)
    bh, bl = _split(b)
    return p, ((ah * bh - p) + ah * bl + al * bh) + al * bl


def dot2_matmul(A, B):
    m, k = A.shape
    s = np.zeros((m, B.shape[1]))
    c = np.zeros_like(s)
    for t in range(k):
        p, e = _two_prod(A[:, t:t + 1], B[t:t + 1, :])
        s, q = _two_sum(s, p)
        c += q + e
    return s + c


def _inputs(n, phi, seed):
    rng = np.random.default_rng(seed)
    A = (rng.random((n, n)) - 0.5) * np.exp(phi * rng.standard_normal((n, n)))
    B = (rng.random((n, n)) - 0.5) * np.exp(phi * rng.standard_normal((n, n)))
    return A, B


@pytest.mark.parametrize("phi", [0.5, 1.0, 2.0])
def test_error_against_moduli_and_fp64_at_default(phi):
    """Below the needed modulus product the CRT wraps around and every entry is
    wrong by about M/2; once M exceeds 2k * 2^106 (the reference's rule,
    ozaki.py:20-29) the result is FP64-accurate, so the curve is a cliff at
    n_mod 22-23 for k = 384 and the default (24) sits past it."""
    n = 384
    A, B = _inputs(n, phi, seed=int(phi * 100))
    ref = dot2_matmul(A, B)
    scale = np.abs(A) @ np.abs(B)
    default = oo.n_moduli(n, 53)
    assert default == 24
    table = {}
    for n_mod in (14, 18, 20, 21, 22, 23, default):
        C = oo.ozaki2_matmul(A, B, n_mod=n_mod)
        rel = np.abs(C - ref) / (EPS * scale)
        table[n_mod] = (float(rel.max()), float(np.median(rel)))
    print(f"\nphi={phi}  n={n}  (error / (eps * |A||B|): max, median)")
    for n_mod, (mx, med) in table.items():
        print(f"  n_mod={n_mod:2d}  max={mx:.3g}  median={med:.3g}")
    for n_mod in (14, 18, 20, 21):  # wrapped: the product of the moduli is too small
        assert table[n_mod][1] > 1e10
    # Past the cliff: the same accuracy with one modulus more or less.
    assert table[23][0] < 1e4 and table[default][0] < 1e4
    assert table[default][1] < 10
    # The reference default: within the split-aware bound, which the reference
    # itself satisfies (k eps |A||B| + scaling truncation of small entries).
    C = oo.ozaki2_matmul(A, B)
    re = np.frexp(np.abs(A).max(axis=1).clip(min=1e-300))[1].astype(np.float64)
    ce = np.frexp(np.abs(B).max(axis=0).clip(min=1e-300))[1].astype(np.float64)
    bound = n * EPS * scale + 2.0 ** -54 * (np.exp2(re)[:, None] * np.abs(B).sum(0)[None, :]
                                            + np.abs(A).sum(1)[:, None] * np.exp2(ce)[None, :])
    assert np.all(np.abs(C - ref) <= bound)
