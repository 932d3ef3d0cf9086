"""The CRT step's exact two-sum.  The reference takes the rounding error of
s = hi + p with TwoSum (crt_reconstruct.cpp:17-26, six operations); the kernels
use Fast2Sum on the two addends ordered by their bit patterns (two operations),
valid because every addend is non-negative.  Both must give the same double at
every step of real accumulations: the CRT weights of every modulus count and
random residues, plus the corner cases of zero addends and exact sums.  Python
floats are IEEE doubles with round-to-nearest, so this is an exact check."""
from __future__ import annotations

import struct

import numpy as np

from oracle import ozaki_oracle as oo


def _bits(x: float) -> int:
    return struct.unpack("<Q", struct.pack("<d", x))[0]


def two_sum(a: float, b: float) -> float:
    s = a + b
    v = s - a
    return (a - (s - v)) + (b - v)


def ordered_fast_two_sum(a: float, b: float) -> float:
    s = a + b
    big, small = (a, b) if _bits(a) > _bits(b) else (b, a)
    return small - (s - big)


def test_fast_two_sum_equals_two_sum_on_crt_accumulations():
    rng = np.random.default_rng(0)
    checked = 0
    for n_mod in range(1, 26):
        moduli = oo.PRIMES[:n_mod]
        wh = oo.crt_weights(moduli)[0]
        for _ in range(400):
            hi = 0.0
            for l, p_l in enumerate(moduli):
                r = float(rng.integers(0, p_l))
                p = r * wh[l]
                t1, t2 = two_sum(hi, p), ordered_fast_two_sum(hi, p)
                assert _bits(t1) == _bits(t2), (n_mod, l, hi, p, t1, t2)
                hi = hi + p
                checked += 1
    for a, b in [(0.0, 0.0), (0.0, 3.0), (3.0, 0.0), (1.0, 2.0 ** -60), (2.0 ** 120, 2.0 ** 120),
                 (1.5, 1.5), (2.0 ** 126 - 2.0 ** 73, 2.0 ** 73)]:
        assert _bits(two_sum(a, b)) == _bits(ordered_fast_two_sum(a, b)), (a, b)
    assert checked > 100_000
