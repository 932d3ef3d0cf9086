"""The reference's CPU path, timed as a baseline.  TEST/BENCH INFRASTRUCTURE ONLY.

Only bench.py (its ``cpu_baseline`` leg and its ``--impl reference`` arm) and
tests use this module.  It runs the reference's own sequence of torch CPU ops
from ``src/fp_emulation/ozaki.py:32-59`` (amax / frexp / ldexp / round, int64
floor-mod residues, torch's int32 batched matmul and ``% p``) and the
reference's own CRT, ``crt_reconstruct.cpp``, compiled from its source into
``oracle/_ref`` (falling back to the C restatement ``crt_oracle.c`` when that
module was never built).  Same arithmetic as the reference, on the host cores.

Large problems are sampled: ``block_time`` computes one r x c block of C
(r full rows of A against c full columns of B) and extrapolates each stage
by how it scales -- the A split with M/r, the B split with N/c, the
per-modulus matmul and the CRT with (M*N)/(r*c).
"""
from __future__ import annotations

import time

import numpy as np
import torch

from oracle import ozaki_oracle as oo


def _crt_module():
    from oracle.build_oracle import load_ref_crt

    try:
        return load_ref_crt()
    except Exception:
        return None


def reference_cpu_path(A: torch.Tensor, B: torch.Tensor, bits: int = 53, n_mod: int | None = None):
    """C = A @ B through the reference's CPU op sequence; returns (C, stage_seconds)."""
    t = [time.perf_counter()]
    if n_mod is None:
        n_mod = oo.n_moduli(A.shape[-1], bits)
    moduli = oo.PRIMES[:n_mod]
    row_exp = A.abs().amax(dim=-1).clamp(min=1e-300).frexp()[1]
    A_int = torch.ldexp(A, bits - row_exp.unsqueeze(-1)).round().to(torch.int64)
    mods64 = torch.tensor(moduli, dtype=torch.int64).view(-1, 1, 1)
    a_res = (A_int.unsqueeze(0) % mods64).to(torch.int8)
    t.append(time.perf_counter())
    col_exp = B.abs().amax(dim=-2).clamp(min=1e-300).frexp()[1]
    B_int = torch.ldexp(B, bits - col_exp.unsqueeze(-2)).round().to(torch.int64)
    b_res = (B_int.unsqueeze(0) % mods64).to(torch.int8)
    t.append(time.perf_counter())
    mods32 = torch.tensor(moduli, dtype=torch.int32).view(-1, 1, 1)
    res = ((a_res.int() @ b_res.int()) % mods32).contiguous()
    t.append(time.perf_counter())
    wh, wm, wl, M_hi, M_lo, inv_M = oo.crt_weights(moduli)
    mod = _crt_module()
    rows, cols = res.shape[1], res.shape[2]
    if mod is not None:
        C = mod.crt_reconstruct(res, torch.tensor(wh, dtype=torch.float64),
                                torch.tensor(wm, dtype=torch.float64),
                                torch.tensor(wl, dtype=torch.float64), M_hi, M_lo, inv_M,
                                row_exp.int().contiguous(), col_exp.int().contiguous(), 2 * bits,
                                rows, cols, n_mod)
    else:
        C = torch.from_numpy(oo.reconstruct(res.numpy(), moduli, bits, row_exp.numpy(), col_exp.numpy()))
    t.append(time.perf_counter())
    return C, [b - a for a, b in zip(t, t[1:])]


def crt_kind() -> str:
    return "reference" if _crt_module() is not None else "port"


def block_time(A_rows: torch.Tensor, B_cols: torch.Tensor, M: int, N: int, bits: int = 53):
    """Time one block and extrapolate to the full M x N product (same K).
    Returns (extrapolated_seconds, block_seconds, stage_seconds)."""
    r, c = A_rows.shape[0], B_cols.shape[1]
    _, st = reference_cpu_path(A_rows, B_cols, bits)
    split_a, split_b, mm, crt = st
    est = split_a * (M / r) + split_b * (N / c) + (mm + crt) * (M * N) / (r * c)
    return est, sum(st), st


def synthetic_block(n: int, r: int, c: int, phi: float, seed: int):
    """r rows of A and c columns of B of the square config-2 inputs,
    (U(0,1) - 0.5) * exp(phi * N(0,1)), generated on the CPU."""
    g = torch.Generator().manual_seed(seed)
    A = (torch.rand(r, n, dtype=torch.float64, generator=g) - 0.5) * \
        torch.exp(phi * torch.randn(r, n, dtype=torch.float64, generator=g))
    B = (torch.rand(n, c, dtype=torch.float64, generator=g) - 0.5) * \
        torch.exp(phi * torch.randn(n, c, dtype=torch.float64, generator=g))
    return A, B


if __name__ == "__main__":
    A, B = synthetic_block(1024, 64, 64, 1.0, 0)
    C, st = reference_cpu_path(A, B)
    want = oo.ozaki2_matmul(A.numpy(), B.numpy())
    print("bit-exact vs oracle:", np.array_equal(C.numpy().view(np.int64), want.view(np.int64)), st)
