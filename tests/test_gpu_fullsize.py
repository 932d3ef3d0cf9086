"""Parity at the benchmark's and the other BASELINE configs' full sizes.

The product is separable: row exponents depend only on A's rows, column
exponents only on B's columns.  So the oracle computes any block C[rows, cols]
exactly from A[rows, :] and B[:, cols], and full-size GPU results are checked
bit for bit on sampled blocks (including extreme rows).  Size-independent
properties are checked on the whole matrix: scaling A by 2 doubles C exactly,
and C(A, B) = C(B^T, A^T)^T bit for bit (the latter runs the two split kernels
on each other's operands).  Accuracy is checked against the split-aware bound
the reference itself satisfies (k eps |A||B| plus the truncation of small
entries relative to their row/column maximum).
"""
from __future__ import annotations

import math

import numpy as np
import pytest

from oracle import ozaki_oracle as oo

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    from fp_emulation import _lib

    _lib.load()
    yield torch
    torch.cuda.empty_cache()
    code = _lib.device_error(clear=True)
    assert code[0] == 0, f"device-side failure recorded: {code}"


def _wide(torch, rows, cols, phi, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    u = torch.rand(rows, cols, dtype=torch.float64, generator=g, device=dev)
    e = torch.randn(rows, cols, dtype=torch.float64, generator=g, device=dev)
    return (u - 0.5) * torch.exp(phi * e)


def _block_parity(C, A, B, rows, cols, bits=53):
    """C[rows][:, cols] (GPU) == oracle product of A[rows, :] and B[:, cols], bitwise."""
    want = oo.ozaki2_matmul(A[rows].cpu().numpy(), B[:, cols].cpu().numpy(), bits=bits)
    got = C[rows][:, cols].cpu().numpy()
    np.testing.assert_array_equal(got.view(np.int64), want.view(np.int64))
    return want


def _split_bound(A, B, rows, cols):
    """k eps |A||B| + 2^-54 (2^re_i sum_t |B_tj| + sum_t |A_it| 2^ce_j) on a block."""
    import torch

    Ab, Bb = A[rows].abs(), B[:, cols].abs()
    k = A.shape[1]
    re = torch.frexp(Ab.amax(dim=1).clamp(min=1e-300))[1].double()
    ce = torch.frexp(Bb.amax(dim=0).clamp(min=1e-300))[1].double()
    return (k * 2.0 ** -53 * (Ab @ Bb)
            + 2.0 ** -54 * (torch.exp2(re)[:, None] * Bb.sum(0)[None, :] + Ab.sum(1)[:, None] * torch.exp2(ce)[None, :]))


def test_config2_n16384_block_parity_and_properties(torch_cuda):
    """BASELINE config 2 at its benchmark point (n = 16384, phi = 1, n_mod = 25)."""
    torch = torch_cuda
    from fp_emulation import ozaki2_int8_matmul

    dev = torch.device("cuda", 0)
    n = 16384
    A = _wide(torch, n, n, 1.0, 11, dev)
    B = _wide(torch, n, n, 1.0, 12, dev)
    C = ozaki2_int8_matmul(A, B)
    rows = torch.tensor([0, 1, 255, 256, 4097, 8191, 12345, 16383])
    cols = torch.cat([torch.arange(0, 16), torch.arange(250, 262), torch.randperm(n)[:200], torch.tensor([n - 1])])
    _block_parity(C, A, B, rows, cols)
    # Exact doubling: 2A has every row exponent one higher and the same integers.
    C2 = ozaki2_int8_matmul(2.0 * A, B)
    assert torch.equal(C2, 2.0 * C)
    del C2
    # Transpose identity, through the other split kernel for each operand.
    Ct = ozaki2_int8_matmul(B.T, A.T)
    assert torch.equal(Ct.T, C)
    del Ct
    # Accuracy against FP64 DGEMM on the block, within the reference's own bound.
    ref = A[rows] @ B[:, cols]
    err = (C[rows][:, cols] - ref).abs()
    assert bool((err <= _split_bound(A, B, rows, cols)).all())


def test_config3_rectangular_rows_scaled(torch_cuda):
    """m = 131072, k = 8192, n = 8192, N(0,1) with 1 % of A's rows x 2^40."""
    torch = torch_cuda
    from fp_emulation import ozaki2_int8_matmul

    dev = torch.device("cuda", 0)
    m, k, n = 131072, 8192, 8192
    g = torch.Generator(device=dev).manual_seed(3)
    A = torch.randn(m, k, dtype=torch.float64, generator=g, device=dev)
    B = torch.randn(k, n, dtype=torch.float64, generator=g, device=dev)
    scaled = torch.randperm(m, generator=torch.Generator().manual_seed(4))[: m // 100]
    A[scaled.to(dev)] *= 2.0 ** 40
    C = ozaki2_int8_matmul(A, B)
    rows = torch.cat([scaled[:6], torch.tensor([0, 1, 65535, 65536, m - 1])])
    cols = torch.cat([torch.arange(0, 8), torch.randperm(n)[:120], torch.tensor([n - 1])])
    _block_parity(C, A, B, rows, cols)
    ref = A[rows] @ B[:, cols]
    assert bool(((C[rows][:, cols] - ref).abs() <= _split_bound(A, B, rows, cols)).all())


def test_config4_converted_mlp(torch_cuda):
    """convert()'ed 6 x Linear(4096, 4096) with tanh, batch 16384;
    every layer's pre-activation is bit-exact against the oracle on a row block."""
    torch = torch_cuda
    from torch import nn

    from fp_emulation import convert

    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    layers = []
    for i in range(6):
        layers.append(nn.Linear(4096, 4096))
        if i < 5:
            layers.append(nn.Tanh())
    model = convert(nn.Sequential(*layers)).to(dev)
    g = torch.Generator(device=dev).manual_seed(5)
    h = torch.randn(16384, 4096, dtype=torch.float64, generator=g, device=dev)
    rows = torch.tensor([0, 7, 8191, 16383])
    with torch.no_grad():
        for layer in model:
            if isinstance(layer, nn.Linear):
                z = layer(h)
                W = layer.weight
                want = oo.ozaki2_matmul(h[rows].cpu().numpy(), W.T.cpu().numpy()) + layer.bias.cpu().numpy()
                np.testing.assert_array_equal(z[rows].cpu().numpy().view(np.int64), want.view(np.int64))
                h = z
            else:
                h = layer(h)
        assert bool(torch.isfinite(h).all())


def _cheb(torch, N, dev):
    """Chebyshev-Gauss-Lobatto points x_j = cos(pi j / N) and the differentiation
    matrix on them (the standard construction; off-diagonal c_i/c_j (-1)^(i+j) /
    (x_i - x_j), diagonal = minus the row sum)."""
    j = torch.arange(N + 1, dtype=torch.float64, device=dev)
    x = torch.cos(math.pi * j / N)
    c = torch.ones(N + 1, dtype=torch.float64, device=dev)
    c[0] = c[N] = 2.0
    c = c * (-1.0) ** j
    dX = x[:, None] - x[None, :]
    D = (c[:, None] / c[None, :]) / (dX + torch.eye(N + 1, dtype=torch.float64, device=dev))
    D = D - torch.diag(D.sum(dim=1))
    return x, D


def test_config5_chebyshev_derivatives(torch_cuda):
    """D and D^2 from N = 2048 Gauss-Lobatto points (entries O(N^2))
    applied to 4096 columns u = sin(pi x a) + 0.1 N(0,1), a ~ U(1, 8)."""
    torch = torch_cuda
    from fp_emulation import ozaki2_int8_matmul

    dev = torch.device("cuda", 0)
    x, D = _cheb(torch, 2048, dev)
    D2 = D @ D
    g = torch.Generator(device=dev).manual_seed(6)
    a = 1.0 + 7.0 * torch.rand(4096, dtype=torch.float64, generator=g, device=dev)
    u = torch.sin(math.pi * x[:, None] * a[None, :]) + 0.1 * torch.randn(2049, 4096, dtype=torch.float64,
                                                                        generator=g, device=dev)
    rows = torch.tensor([0, 1, 1024, 2047, 2048])
    cols = torch.arange(0, 4096, 37)
    for M in (D, D2):
        Cm = ozaki2_int8_matmul(M, u)
        _block_parity(Cm, M, u, rows, cols)
        ref = M[rows] @ u[:, cols]
        assert bool(((Cm[rows][:, cols] - ref).abs() <= _split_bound(M, u, rows, cols)).all())
