"""Pin the oracle to the reference: every golden fixture, bit for bit.

The fixtures in tests/golden/ were produced by running the reference's own CPU
path (tests/golden/make_golden.py).  These tests need no GPU.
"""
from __future__ import annotations

import hashlib
import math

import numpy as np
import pytest

from conftest import compensated_matmul, golden_names, load_golden
from oracle import ozaki_oracle as oo


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _check_stage(g, key, arr):
    assert tuple(arr.shape) == tuple(g[f"{key}_shape"]), key
    assert _sha(arr.astype(g[f"{key}_dtype"].item().decode())) == g[f"{key}_sha256"].item().decode(), key


@pytest.mark.parametrize("name", golden_names())
def test_oracle_matches_reference_stages(name):
    g = load_golden(name)
    bits, n_mod = int(g["bits"]), int(g["n_mod"])
    A, B = g["A"], g["B"]
    assert oo.n_moduli(A.shape[1], bits) == n_mod
    C, st = oo.ozaki2_matmul(A, B, bits=bits, stages=True)
    np.testing.assert_array_equal(st["row_exp"], g["row_exp"])
    np.testing.assert_array_equal(st["col_exp"], g["col_exp"])
    if "A_int" in g:
        np.testing.assert_array_equal(st["A_int"], g["A_int"])
        np.testing.assert_array_equal(st["B_int"], g["B_int"])
    _check_stage(g, "a_res", st["a_res"])
    _check_stage(g, "b_res", st["b_res"])
    raw = oo.matmul_residues_raw(st["a_res"], st["b_res"])
    _check_stage(g, "raw", raw.astype(np.int32))
    _check_stage(g, "res", st["res"])
    # Final float64 result of _reconstruct: bit-identical.
    np.testing.assert_array_equal(C.view(np.int64), g["C64"].view(np.int64))


def test_moduli_table():
    """n_mod 24 for k <= 4096 and 25 for 8192 <= k <= 131072 (ozaki.py:20-29)."""
    assert [oo.n_moduli(k, 53) for k in (256, 1024, 4096)] == [24, 24, 24]
    assert [oo.n_moduli(k, 53) for k in (8192, 16384, 131072)] == [25, 25, 25]
    assert oo.n_moduli(16, 53) == 23
    assert [oo.n_moduli(4096, b) for b in (24, 11, 8)] == [15, 10, 9]
    with pytest.raises(ValueError):
        oo.n_moduli(2 ** 60, 53)


def test_crt_weights_exact():
    """(wh + wm + wl) equals the exact CRT weight to well below one unit."""
    for n in (8, 14, 23, 24, 25):
        mods = oo.PRIMES[:n]
        M = math.prod(mods)
        wh, wm, wl, M_hi, M_lo, inv_M = oo.crt_weights(mods)
        for m, a, b, c in zip(mods, wh, wm, wl):
            Mi = M // m
            w = Mi * pow(Mi, -1, m)
            assert w % m == 1 and w % (M // m) == 0
            assert abs(int(a) + int(b) + int(c) - w) <= 1
        # M is carried as a double-double (about 106 bits), not exactly.
        assert abs(int(M_hi) + int(M_lo) - M) <= 2 ** max(0, M.bit_length() - 106)


def test_oracle_vs_compiled_reference_crt():
    """The C restatement and the reference's own crt_reconstruct.cpp (compiled
    from its source into oracle/_ref) agree bit for bit."""
    from oracle.build_oracle import load_ref_crt

    ref = load_ref_crt()
    if ref is None:
        pytest.skip("reference CRT module not built (oracle/_ref)")
    import torch

    g = load_golden("cfg1_256")
    C, st = oo.ozaki2_matmul(g["A"], g["B"], stages=True)
    wh, wm, wl, M_hi, M_lo, inv_M = oo.crt_weights(st["moduli"])
    out = ref.crt_reconstruct(
        torch.from_numpy(st["res"]).contiguous(), torch.tensor(wh, dtype=torch.float64),
        torch.tensor(wm, dtype=torch.float64), torch.tensor(wl, dtype=torch.float64),
        M_hi, M_lo, inv_M, torch.from_numpy(st["row_exp"]), torch.from_numpy(st["col_exp"]),
        106, 256, 256, len(st["moduli"])).numpy()
    np.testing.assert_array_equal(out.view(np.int64), C.view(np.int64))


def test_oracle_accuracy_vs_compensated():
    """Reference tests/test_ozaki.py:6-14: < 1e-14 from the compensated product."""
    g = load_golden("ref_accuracy_16")
    C = oo.ozaki2_matmul(g["A"], g["B"])
    assert np.max(np.abs(C - compensated_matmul(g["A"], g["B"]))) < 1e-14


def test_oracle_u8_residues_same_as_int32():
    g = load_golden("wide_phi2.0_64x96x80")
    C, st = oo.ozaki2_matmul(g["A"], g["B"], stages=True)
    C8 = oo.reconstruct(st["res"].astype(np.uint8), st["moduli"], 53, st["row_exp"], st["col_exp"])
    np.testing.assert_array_equal(C8.view(np.int64), C.view(np.int64))
