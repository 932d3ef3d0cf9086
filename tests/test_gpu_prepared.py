"""Prepared (cached-split) operands on the GPU: products with a prepared left
operand (the Chebyshev D of ``D @ u``), a prepared right operand, or both are
bit-identical to the CPU oracle and to the unprepared product; the split is
reused while the operand is unchanged and redone after an in-place update; the
backward products through the prepared transposes give the oracle's gradients
(ozaki.py:132-136: grad_B = A^T @ grad)."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import ozaki_oracle as oo

pytestmark = pytest.mark.gpu


def cheb(N):
    """Chebyshev-Gauss-Lobatto points and differentiation matrix on N+1 points
    (the construction of the reference's DT-PINN notebook, written for numpy)."""
    x = np.cos(np.pi * np.arange(N + 1) / N)
    c = np.ones(N + 1)
    c[0] = c[N] = 2.0
    c = c * (-1.0) ** np.arange(N + 1)
    dX = x[:, None] - x[None, :]
    D = (c[:, None] / c[None, :]) / (dX + np.eye(N + 1))
    return x, D - np.diag(D.sum(axis=1))


def _fields(x, cols, seed):
    rng = np.random.default_rng(seed)
    a = rng.uniform(1, 8, cols)
    return np.sin(np.pi * x[:, None] * a[None, :]) + 0.1 * rng.standard_normal((x.size, cols))


def _same(got, want):
    np.testing.assert_array_equal(np.asarray(got).view(np.int64), np.asarray(want).view(np.int64))


def test_prepared_left_operand_is_exact_and_reused():
    import torch

    from fp_emulation import ozaki2_int8_matmul, prepare_operand

    x, D = cheb(300)
    D2 = D @ D
    dev = torch.device("cuda", 0)
    Dp = prepare_operand(torch.from_numpy(D).to(dev), "left")
    D2p = prepare_operand(torch.from_numpy(D2).to(dev), "left")
    for seed in (1, 2):  # a new field every "epoch"; the operators' splits are reused
        u = _fields(x, 129, seed)
        ut = torch.from_numpy(u).to(dev)
        Du = ozaki2_int8_matmul(Dp, ut)
        D2u = ozaki2_int8_matmul(D2p, ut)
        _same(Du.cpu().numpy(), oo.ozaki2_matmul(D, u))
        _same(D2u.cpu().numpy(), oo.ozaki2_matmul(D2, u))
        _same(Du.cpu().numpy(), ozaki2_int8_matmul(Dp.tensor, ut).cpu().numpy())
        if seed == 1:
            first = Dp._split[1]
        else:
            assert Dp._split[1] is first, "an unchanged operand must keep its split"
    Dp.tensor.mul_(2.0)  # in place: bumps the version, the split is redone
    Du = ozaki2_int8_matmul(Dp, ut)
    assert Dp._split[1] is not first
    _same(Du.cpu().numpy(), oo.ozaki2_matmul(2.0 * D, u))


@pytest.mark.parametrize("which", ["right", "both"])
def test_prepared_right_and_both(which):
    import torch

    from fp_emulation import ozaki2_int8_matmul, prepare_operand

    rng = np.random.default_rng(7)
    A = (rng.random((190, 333)) - 0.5) * np.exp(rng.standard_normal((190, 333)))
    B = (rng.random((333, 270)) - 0.5) * np.exp(rng.standard_normal((333, 270)))
    dev = torch.device("cuda", 0)
    At, Bt = torch.from_numpy(A).to(dev), torch.from_numpy(B).to(dev)
    left = prepare_operand(At, "left") if which == "both" else At
    C = ozaki2_int8_matmul(left, prepare_operand(Bt, "right"))
    _same(C.cpu().numpy(), oo.ozaki2_matmul(A, B))
    # A transposed view prepared as the right operand (strided split).
    Ct = ozaki2_int8_matmul(Bt.T, prepare_operand(At.T, "right"))
    _same(Ct.cpu().numpy(), oo.ozaki2_matmul(B.T, A.T))


def test_backward_through_prepared_operator():
    """u requires grad, D is a prepared constant: u.grad = D^T @ G through D's
    prepared transpose, equal to the oracle and to the unprepared backward."""
    import torch

    from fp_emulation import ozaki2_int8_matmul, prepare_operand

    x, D = cheb(200)
    u = _fields(x, 64, 3)
    G = np.random.default_rng(9).standard_normal((201, 64))
    dev = torch.device("cuda", 0)
    Dp = prepare_operand(torch.from_numpy(D).to(dev), "left")
    ut = torch.from_numpy(u).to(dev).requires_grad_(True)
    out = ozaki2_int8_matmul(Dp, ut)
    out.backward(torch.from_numpy(G).to(dev))
    _same(ut.grad.cpu().numpy(), oo.ozaki2_matmul(D.T, G))
    assert Dp.T._split is not None, "the backward product must use the prepared transpose"
    u2 = torch.from_numpy(u).to(dev).requires_grad_(True)
    ozaki2_int8_matmul(torch.from_numpy(D).to(dev), u2).backward(torch.from_numpy(G).to(dev))
    assert torch.equal(u2.grad, ut.grad)


def test_prepared_float32_matches_unprepared():
    import torch

    from fp_emulation import ozaki2_int8_matmul, prepare_operand

    rng = np.random.default_rng(11)
    A = torch.from_numpy(rng.standard_normal((64, 300))).float().cuda()
    B = torch.from_numpy(rng.standard_normal((300, 80))).float().cuda()
    C = ozaki2_int8_matmul(prepare_operand(A, "left"), B)
    assert C.dtype == torch.float32
    assert torch.equal(C, ozaki2_int8_matmul(A, B))


def test_prepared_side_mismatch_raises():
    import torch

    from fp_emulation import ozaki2_int8_matmul, prepare_operand

    A = torch.randn(8, 8, dtype=torch.float64, device="cuda")
    with pytest.raises(ValueError):
        ozaki2_int8_matmul(prepare_operand(A, "right"), A)
    with pytest.raises(ValueError):
        ozaki2_int8_matmul(A, prepare_operand(A, "left"))
