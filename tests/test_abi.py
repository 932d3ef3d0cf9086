"""C-ABI and host-logic tests that need no GPU.

* libfpemu.so loads and exports every symbol include/fpemu.h declares;
* its host-side planning (moduli, CRT weights, int32 limit) equals the oracle;
* the integer tricks the kernels rely on (magic-number division, the 3-limb
  fold of 53-bit integers) are exact, checked here over their input ranges;
* the Python layer raises the reference's exceptions before touching a GPU.
"""
from __future__ import annotations

import ctypes
import re

import numpy as np
import pytest

from conftest import REPO
from oracle import ozaki_oracle as oo

HEADER = REPO / "include" / "fpemu.h"


def _lib():
    from fp_emulation import _lib as L

    return L.load()


def test_library_exports_every_declared_symbol():
    names = set(re.findall(r"\b(fpemu_[a-z0-9_]+)\s*\(", HEADER.read_text()))
    assert len(names) >= 14
    lib = _lib()
    for name in sorted(names):
        assert hasattr(lib, name), name
    from fp_emulation import _lib as L

    assert names == set(L.SIGNATURES), "ctypes signatures out of sync with the header"
    assert lib.fpemu_abi_version() == 1


@pytest.mark.parametrize("bits", [53, 24, 11, 8])
def test_plan_moduli_matches_reference_rule(bits):
    lib = _lib()
    n = ctypes.c_int()
    mods = (ctypes.c_int32 * 32)()
    for k in [1, 2, 16, 20, 255, 256, 1000, 4096, 4097, 8191, 8192, 16384, 131072, 214748]:
        assert lib.fpemu_plan_moduli(k, bits, ctypes.byref(n), mods) == 0
        assert n.value == oo.n_moduli(k, bits), (k, bits)
        assert list(mods[: n.value]) == oo.PRIMES[: n.value]
    assert lib.fpemu_plan_moduli(2 ** 60, 53, ctypes.byref(n), None) == 2  # FPEMU_ERR_NO_MODULI


def test_crt_weights_bit_identical_to_reference_formula():
    lib = _lib()
    for n_mod in range(1, 26):
        arr = [(ctypes.c_double * n_mod)() for _ in range(3)]
        sc = [ctypes.c_double() for _ in range(3)]
        assert lib.fpemu_crt_weights(n_mod, *arr, *[ctypes.byref(s) for s in sc]) == 0
        ref = oo.crt_weights(oo.PRIMES[:n_mod])
        for got, want in zip(arr, ref[:3]):
            np.testing.assert_array_equal(np.array(list(got)).view(np.int64), np.array(want).view(np.int64))
        for got, want in zip(sc, ref[3:]):
            assert np.float64(got.value).view(np.int64) == np.float64(want).view(np.int64)
    assert lib.fpemu_crt_weights(26, *arr, *[ctypes.byref(s) for s in sc]) == 3  # FPEMU_ERR_UNSUPPORTED


def test_max_k_is_the_int32_limit():
    lib = _lib()
    assert lib.fpemu_max_k(25) == (2 ** 31 - 1) // (100 * 100)
    assert lib.fpemu_max_k(24) == (2 ** 31 - 1) // (96 * 96)


def _mod_consts(p):
    s = p.bit_length() - 1
    return s, -(-(1 << (32 + s)) // p)


def test_magic_division_exact_below_2_31():
    """floor(n/p) == (n * magic) >> (32 + s) for every n < 2^31 (checked on a dense
    set: every multiple-of-p boundary neighbourhood plus random values)."""
    rng = np.random.default_rng(0)
    for p in oo.PRIMES[:25]:
        s, magic = _mod_consts(p)
        assert magic < 2 ** 32
        q = np.arange(0, (2 ** 31 - 1) // p + 1, max(1, ((2 ** 31) // p) // 200_000), dtype=np.uint64)
        n = np.concatenate([q * p, q * p + p - 1, q * p + 1,
                            rng.integers(0, 2 ** 31, 200_000, dtype=np.uint64),
                            np.array([2 ** 31 - 1, 0, p - 1], dtype=np.uint64)])
        n = n[n < 2 ** 31]
        got = ((n * np.uint64(magic)) >> np.uint64(32)) >> np.uint64(s)
        np.testing.assert_array_equal(got, n // np.uint64(p))


def test_fold_residues_exact():
    """The split kernel's residue path: |v| = a*2^36 + b*2^18 + c, fold with
    2^36 mod p and 2^18 mod p, negate as p*2^24 - t, reduce by magic division;
    must equal Python's floor-mod for |v| <= 2^53."""
    rng = np.random.default_rng(1)
    v = np.concatenate([rng.integers(-(2 ** 53), 2 ** 53 + 1, 300_000, dtype=np.int64),
                        np.array([0, 1, -1, 2 ** 53, -(2 ** 53), 2 ** 53 - 1, -(2 ** 36), 2 ** 18 - 1],
                                 dtype=np.int64)])
    u = np.abs(v).astype(np.uint64)
    a, b, c = u >> np.uint64(36), (u >> np.uint64(18)) & np.uint64(0x3FFFF), u & np.uint64(0x3FFFF)
    for p in oo.PRIMES[:25]:
        s, magic = _mod_consts(p)
        t = a * np.uint64((1 << 36) % p) + b * np.uint64((1 << 18) % p) + c
        assert int(t.max()) < p << 24
        t = np.where(v < 0, np.uint64(p << 24) - t, t)
        assert int(t.max()) < 2 ** 31
        r = t - (((t * np.uint64(magic)) >> np.uint64(32 + s)) * np.uint64(p))
        np.testing.assert_array_equal(r.astype(np.int64), np.mod(v, p))


def test_python_layer_errors_without_gpu():
    import torch

    from fp_emulation import ozaki2_int8_matmul
    from fp_emulation.ozaki import _crt_weights, _n_moduli

    assert _n_moduli(16384, 53) == 25
    assert _crt_weights(oo.PRIMES[:24]) == tuple(oo.crt_weights(oo.PRIMES[:24])) or \
        list(_crt_weights(oo.PRIMES[:24])) == list(oo.crt_weights(oo.PRIMES[:24]))
    with pytest.raises(ValueError):
        _n_moduli(2 ** 60, 53)
    with pytest.raises(TypeError):  # ozaki.py:99-104: dtype first
        ozaki2_int8_matmul(torch.ones(2, 2, dtype=torch.int32), torch.ones(2, 2, dtype=torch.int32))
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        ozaki2_int8_matmul(torch.ones(2, 2, dtype=torch.float64), torch.ones(2, 2, dtype=torch.float64))


# The split kernel's residue path (split_kernels.cuh): the scaled value x (an
# integer-valued double, |x| <= 2^53) is reduced modulo 5 prime groups in FP64
# -- q = floor(x * RN(1/P)), r0 = fma(-q, P, x) (exact), y = low word of
# r0 + (2P + 2^52) -- and each prime then takes y mod p by magic division.
PRIME_GROUPS = [(0, 8), (8, 13), (13, 17), (17, 21), (21, 25)]


def test_prime_groups_cover_moduli_and_fit():
    assert PRIME_GROUPS[0][0] == 0 and PRIME_GROUPS[-1][1] == 25
    for (a, b), (c, _) in zip(PRIME_GROUPS, PRIME_GROUPS[1:]):
        assert b == c
    for a, b in PRIME_GROUPS:
        P = int(np.prod(oo.PRIMES[a:b], dtype=object))
        assert P < 2 ** 27  # so r0 + 2P stays in [P, 4P) < 2^29 < 2^31


def test_group_reduction_exact():
    rng = np.random.default_rng(2)
    x = np.concatenate([rng.integers(-(2 ** 53), 2 ** 53 + 1, 200_000, dtype=np.int64),
                        np.array([0, 1, -1, 2 ** 53, -(2 ** 53), 2 ** 52 + 1, -(2 ** 52) - 1], dtype=np.int64)])
    xd = x.astype(np.float64)
    assert np.all(xd.astype(np.int64) == x)
    for a, b in PRIME_GROUPS:
        P = int(np.prod(oo.PRIMES[a:b], dtype=object))
        invP = np.float64(1.0) / np.float64(P)
        q = np.floor(xd * invP)                       # FP64 multiply (RN), floor
        r0 = x - q.astype(np.int64) * P               # the fma is exact: integer arithmetic
        assert np.all(r0 >= -P) and np.all(r0 < 2 * P)
        y = r0 + 2 * P                                # low word of r0 + (2P + 2^52)
        assert np.all(y >= P) and np.all(y < 2 ** 31)
        for p in oo.PRIMES[a:b]:
            s, magic = _mod_consts(p)
            yu = y.astype(np.uint64)
            r = yu - ((yu * np.uint64(magic)) >> np.uint64(32 + s)) * np.uint64(p)
            np.testing.assert_array_equal(r.astype(np.int64), np.mod(x, p))


def test_transport_and_fusion_entry_points_validate_on_the_host():
    """The fused-epilogue entry points reject bad arguments before any CUDA call."""
    from fp_emulation import _lib as L

    lib = _lib()
    # Output dtype codes other than FPEMU_C_F64 / FPEMU_C_F32 are refused.
    st = lib.fpemu_gemm_crt_ex(4, 4, 4, 24, None, None, 16, 64, None, None, 53, None, 4, 7, None, 0, None, 0, None)
    assert st == L.FPEMU_ERR_INVALID
    assert b"c_dtype" in lib.fpemu_last_error()


def test_watch_loads_the_library_without_deadlock():
    """The first library call of a process may be the one that arms the error
    watch: _lib.watch must load the library itself without waiting on its own
    lock.  Checked in a fresh process with the CUDA entry point replaced."""
    import subprocess
    import sys
    import textwrap

    code = textwrap.dedent(f"""
        import sys, threading
        sys.path.insert(0, {str(REPO / 'fp-emulation_b200')!r})
        from fp_emulation import _lib
        assert _lib._lib is None
        calls = []
        real_load = _lib.load

        def load():
            lib = real_load()
            class Shim:
                def __getattr__(self, name):
                    return getattr(lib, name)
                def fpemu_watch_errors(self):
                    calls.append(1)
                    return 0
            return Shim()

        _lib.load = load
        t = threading.Thread(target=_lib.watch, args=(0,), daemon=True)
        t.start()
        t.join(20)
        assert not t.is_alive(), "watch() deadlocked"
        assert calls == [1] and 0 in _lib._watched
        print("ok")
    """)
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=60)
    assert res.returncode == 0 and res.stdout.strip() == "ok", res.stdout + res.stderr


def test_prepared_operand_validates_on_the_host():
    """prepare_operand keeps the public op's rules: CUDA tensors only, 2-D,
    float dtypes (TypeError otherwise), and a side of 'left' or 'right'."""
    import pytest
    import torch

    from fp_emulation import prepare_operand

    with pytest.raises(ValueError):
        prepare_operand(torch.zeros(2, 2, dtype=torch.float64), "middle")
    with pytest.raises(TypeError):
        prepare_operand(torch.zeros(2, 2, dtype=torch.int32), "left")
    with pytest.raises(RuntimeError, match="CUDA"):
        prepare_operand(torch.zeros(2, 2, dtype=torch.float64), "left")
    with pytest.raises(RuntimeError):
        prepare_operand(torch.zeros(2, dtype=torch.float64), "left")
