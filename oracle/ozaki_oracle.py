"""CPU restatement of the reference's Ozaki scheme II path (the parity oracle).

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this module;
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its CPU
baseline leg and its ``--impl reference`` arm) load it, and only as the
checker or as the timed CPU baseline.

Each function restates one step of ``src/fp_emulation/ozaki.py`` of
thezettascale/fp-emulation and names the lines it follows.  Integer and byte
work is numpy; the CRT arithmetic is the C file ``crt_oracle.c`` (numpy has no
fused multiply-add, and the reference's CRT relies on ``fma``).

Parity is pinned: ``tests/golden/`` holds fixtures produced by running the
reference itself in the build container (``tests/golden/make_golden.py``), and
``tests/test_oracle_golden.py`` checks this module against every one of them
bit for bit.
"""
from __future__ import annotations

import ctypes
import math
import os
from pathlib import Path

import numpy as np

# ozaki.py:6-9 -- the odd primes the reference draws moduli from, in order.
PRIMES = [
    3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37, 41, 43, 47, 53,
    59, 61, 67, 71, 73, 79, 83, 89, 97, 101, 103, 107, 109, 113, 127,
]

# ozaki.py:12-17 -- mantissa bits per input dtype (keys are numpy/torch names).
PRECISION_BITS = {"float16": 11, "bfloat16": 8, "float32": 24, "float64": 53}

_HERE = Path(__file__).resolve().parent
_LIB = None


def _lib():
    """Load the compiled C half of the oracle (built by oracle/build_oracle.py)."""
    global _LIB
    if _LIB is None:
        path = _HERE / "_build" / "libcrt_oracle.so"
        if not path.exists():
            from oracle.build_oracle import build_oracle_lib

            build_oracle_lib()
        lib = ctypes.CDLL(str(path))
        i64, i32, dbl, vp = ctypes.c_int64, ctypes.c_int, ctypes.c_double, ctypes.c_void_p
        for name in ("oracle_crt_reconstruct", "oracle_crt_reconstruct_u8"):
            f = getattr(lib, name)
            f.restype = None
            f.argtypes = [vp, vp, vp, vp, dbl, dbl, dbl, vp, vp, i32, vp, i64, i64, i32]
        lib.oracle_residues.restype = None
        lib.oracle_residues.argtypes = [vp, i64, vp, i32, vp]
        _LIB = lib
    return _LIB


def n_moduli(k: int, bits: int) -> int:
    """ozaki.py:20-29: fewest leading primes whose product exceeds 2*k*2^(2*bits)."""
    target = 2 * k * (2 ** (2 * bits))
    prod = 1
    for i, p in enumerate(PRIMES):
        prod *= p
        if prod > target:
            return i + 1
    raise ValueError(f"not enough primes for inner dim {k}, bits {bits}")


def scale_to_int(A: np.ndarray, B: np.ndarray, bits: int):
    """ozaki.py:32-38.

    row_exp[i] = frexp(max(max_j |A_ij|, 1e-300)).exponent, and
    A_int = round_half_even(A * 2^(bits - row_exp[i])) as int64; the same for
    the columns of B.  ``np.ldexp`` is exact like ``torch.ldexp`` on float64,
    and ``np.rint`` rounds half to even like ``torch.round``.
    """
    row_max = np.maximum(np.abs(A).max(axis=-1, initial=0.0), 1e-300)
    col_max = np.maximum(np.abs(B).max(axis=-2, initial=0.0), 1e-300)
    row_exp = np.frexp(row_max)[1].astype(np.int32)
    col_exp = np.frexp(col_max)[1].astype(np.int32)
    A_int = np.rint(np.ldexp(A, (bits - row_exp)[:, None])).astype(np.int64)
    B_int = np.rint(np.ldexp(B, (bits - col_exp)[None, :])).astype(np.int64)
    return A_int, B_int, row_exp, col_exp


def residues(X_int: np.ndarray, moduli) -> np.ndarray:
    """ozaki.py:41-46: floor-mod residues, int8 [n_mod, *X.shape], values in [0, p)."""
    X = np.ascontiguousarray(X_int, dtype=np.int64)
    out = np.empty((len(moduli),) + X.shape, dtype=np.int8)
    mods = np.asarray(moduli, dtype=np.int32)
    _lib().oracle_residues(X.ctypes.data, X.size, mods.ctypes.data, len(moduli), out.ctypes.data)
    return out


def matmul_residues_raw(a_res: np.ndarray, b_res: np.ndarray) -> np.ndarray:
    """Raw per-modulus products a_res[l] @ b_res[l] as int64 (the int32 values of
    ``a_res.int() @ b_res.int()``, ozaki.py:59, before the ``% p``).

    Computed with float64 BLAS: every partial sum is an integer below
    k*127^2 < 2^53, so the result is exact in any summation order.
    """
    a = a_res.astype(np.float64)
    b = b_res.astype(np.float64)
    return np.matmul(a, b).astype(np.int64)


def matmul_residues(a_res: np.ndarray, b_res: np.ndarray, moduli) -> np.ndarray:
    """ozaki.py:49-59 (CPU branch): (a_l @ b_l) mod p_l, int32 [n_mod, M, N]."""
    raw = matmul_residues_raw(a_res, b_res)
    mods = np.asarray(moduli, dtype=np.int64).reshape(-1, 1, 1)
    return np.mod(raw, mods).astype(np.int32)


def crt_weights(moduli):
    """ozaki.py:62-80: CRT weights split into (hi, mid, lo) doubles, and M split
    into (M_hi, M_lo) with inv_M = 1/float(M).  Python integers are exact."""
    M = math.prod(moduli)
    wh, wm, wl = [], [], []
    for m in moduli:
        Mi = M // m
        w = Mi * pow(Mi, -1, m)
        hi = float(w)
        r = w - int(hi)
        mid = float(r)
        lo = float(r - int(mid))
        wh.append(hi)
        wm.append(mid)
        wl.append(lo)
    M_hi = float(M)
    M_lo = float(M - int(M_hi))
    inv_M = 1.0 / float(M)
    return wh, wm, wl, M_hi, M_lo, inv_M


def reconstruct(res: np.ndarray, moduli, bits: int, row_exp, col_exp) -> np.ndarray:
    """ozaki.py:83-92 -> crt_reconstruct.cpp:6-38 (through crt_oracle.c).

    ``res`` is [n_mod, M, N] int32 or uint8 residues in [0, p).
    """
    n_mod, rows, cols = res.shape
    wh, wm, wl, M_hi, M_lo, inv_M = crt_weights(moduli)
    wh = np.asarray(wh, dtype=np.float64)
    wm = np.asarray(wm, dtype=np.float64)
    wl = np.asarray(wl, dtype=np.float64)
    re = np.ascontiguousarray(row_exp, dtype=np.int32)
    ce = np.ascontiguousarray(col_exp, dtype=np.int32)
    out = np.empty((rows, cols), dtype=np.float64)
    if res.dtype == np.uint8:
        r = np.ascontiguousarray(res)
        fn = _lib().oracle_crt_reconstruct_u8
    else:
        r = np.ascontiguousarray(res, dtype=np.int32)
        fn = _lib().oracle_crt_reconstruct
    fn(r.ctypes.data, wh.ctypes.data, wm.ctypes.data, wl.ctypes.data, M_hi, M_lo, inv_M,
       re.ctypes.data, ce.ctypes.data, 2 * bits, out.ctypes.data, rows, cols, n_mod)
    return out


def ozaki2_matmul(A: np.ndarray, B: np.ndarray, bits: int = 53, n_mod: int | None = None,
                  stages: bool = False):
    """ozaki.py:95-119 for float64 arrays (the caller upcasts other dtypes and
    picks ``bits`` from the original dtype, as ozaki.py:97-107 does).

    ``n_mod`` overrides the modulus count (the reference always uses
    ``n_moduli(k, bits)``); ``stages=True`` also returns every intermediate.
    """
    A = np.asarray(A, dtype=np.float64)
    B = np.asarray(B, dtype=np.float64)
    if n_mod is None:
        n_mod = n_moduli(A.shape[-1], bits)
    moduli = PRIMES[:n_mod]
    A_int, B_int, row_exp, col_exp = scale_to_int(A, B, bits)
    a_res = residues(A_int, moduli)
    b_res = residues(B_int, moduli)
    res = matmul_residues(a_res, b_res, moduli)
    C = reconstruct(res, moduli, bits, row_exp, col_exp)
    if not stages:
        return C
    return C, dict(A_int=A_int, B_int=B_int, row_exp=row_exp, col_exp=col_exp, a_res=a_res,
                   b_res=b_res, res=res, moduli=moduli)


def cpu_threads() -> int:
    """Threads the C half of the oracle may use (OpenMP reads OMP_NUM_THREADS)."""
    return int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
