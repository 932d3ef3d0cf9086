"""The epilogue fusions and the static-operand cache against the oracle.

* float32 inputs: the kernel writes the float result directly; it must equal
  the reference's float64 result rounded by ``.to(torch.float32)``
  (ozaki.py:117-118).
* ``nn.Linear`` without autograd recording: the bias add is fused into the
  epilogue; the result must equal the reference's ``matmul + bias`` (nn.py:18-21),
  i.e. the oracle's product plus the bias in float64, bit for bit.
* ``cache_weight_residues``: the weight is split once and reused; an in-place
  update of the weight invalidates the cache.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import ozaki_oracle as oo

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["fused", "split"], autouse=True)
def gemm_path(request, monkeypatch):
    """Every test of this module runs on both forms of the GEMM + CRT stage: the
    fused kernel and the split form (spread residue GEMM, then the CRT kernel);
    FPEMU_GEMM_PATH forces one where the size would pick the other."""
    monkeypatch.setenv("FPEMU_GEMM_PATH", request.param)
    return request.param


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    from fp_emulation import _lib

    _lib.load()
    yield torch
    code = _lib.device_error(clear=True)
    assert code[0] == 0, f"device-side failure recorded: {code}"


def _case(seed, m, k, n):
    rng = np.random.default_rng(seed)
    A = (rng.random((m, k)) - 0.5) * np.exp(1.5 * rng.standard_normal((m, k)))
    B = (rng.random((k, n)) - 0.5) * np.exp(1.5 * rng.standard_normal((k, n)))
    return A, B


@pytest.mark.parametrize("m,k,n", [(1, 5, 3), (129, 300, 257), (300, 1000, 77)])
def test_float32_output_is_the_rounded_float64_result(torch_cuda, m, k, n):
    torch = torch_cuda
    from fp_emulation import ozaki2_int8_matmul

    A, B = _case(m + 3 * k + 7 * n, m, k, n)
    A32, B32 = A.astype(np.float32), B.astype(np.float32)
    got = ozaki2_int8_matmul(torch.from_numpy(A32).cuda(), torch.from_numpy(B32).cuda())
    assert got.dtype == torch.float32
    want = oo.ozaki2_matmul(A32.astype(np.float64), B32.astype(np.float64), bits=24).astype(np.float32)
    np.testing.assert_array_equal(got.cpu().numpy().view(np.int32), want.view(np.int32))


def test_forward_bias_fusion_float32_and_float64(torch_cuda):
    torch = torch_cuda
    from fp_emulation.ozaki import _ozaki2_forward

    A, B = _case(11, 70, 200, 90)
    bias = np.random.default_rng(12).standard_normal(90)
    for dt, np_dt, bits in ((torch.float64, np.float64, 53), (torch.float32, np.float32, 24)):
        Ad, Bd = torch.from_numpy(A).to(dt).cuda(), torch.from_numpy(B).to(dt).cuda()
        bd = torch.from_numpy(bias).to(dt).cuda()
        got = _ozaki2_forward(Ad, Bd, bias=bd).cpu().numpy()
        prod = oo.ozaki2_matmul(Ad.double().cpu().numpy(), Bd.double().cpu().numpy(), bits=bits).astype(np_dt)
        want = prod + bias.astype(np_dt)
        assert got.dtype == np_dt
        np.testing.assert_array_equal(got, want)


def _linear(torch, seed, in_f, out_f, cache):
    from fp_emulation.nn import Linear

    torch.manual_seed(seed)
    lin = Linear(in_f, out_f, cache_weight_residues=cache).cuda()
    return lin


@pytest.mark.parametrize("cache", [False, True])
def test_linear_fused_bias_matches_reference_order(torch_cuda, cache):
    torch = torch_cuda
    lin = _linear(torch, 0, 300, 130, cache)
    x = torch.randn(4, 50, 300, dtype=torch.float64, generator=torch.Generator().manual_seed(1)).cuda()
    with torch.no_grad():
        y = lin(x)
    W = lin.weight.detach().cpu().numpy()
    b = lin.bias.detach().cpu().numpy()
    want = oo.ozaki2_matmul(x.reshape(-1, 300).cpu().numpy(), W.T) + b
    np.testing.assert_array_equal(y.reshape(-1, 130).cpu().numpy().view(np.int64), want.view(np.int64))
    # The autograd path (unfused: product, then torch's add) gives the same bits.
    y_grad = lin(x)
    assert y_grad.requires_grad
    assert torch.equal(y_grad.detach(), y)


def test_linear_weight_cache_reuse_and_invalidation(torch_cuda):
    torch = torch_cuda
    lin = _linear(torch, 3, 257, 65, True)
    x = torch.randn(33, 257, dtype=torch.float64, generator=torch.Generator().manual_seed(4)).cuda()
    with torch.no_grad():
        y1 = lin(x)
        first = lin._weight_op[1]._split[1]
        y2 = lin(x)
        assert lin._weight_op[1]._split[1] is first, "an unchanged weight must reuse its split"
        assert torch.equal(y1, y2)
        lin.weight.mul_(-0.5)  # in place: bumps the version
        y3 = lin(x)
        assert lin._weight_op[1]._split[1] is not first, "an in-place update must re-split the weight"
    W = lin.weight.detach().cpu().numpy()
    want = oo.ozaki2_matmul(x.cpu().numpy(), W.T) + lin.bias.detach().cpu().numpy()
    np.testing.assert_array_equal(y3.cpu().numpy().view(np.int64), want.view(np.int64))


def test_converted_mlp_cached_equals_uncached(torch_cuda):
    torch = torch_cuda
    from torch import nn

    from fp_emulation import convert

    def build(cache):
        torch.manual_seed(7)
        layers = []
        for i in range(3):
            layers.append(nn.Linear(96, 96))
            if i < 2:
                layers.append(nn.Tanh())
        return convert(nn.Sequential(*layers), cache_weight_residues=cache).cuda()

    x = torch.randn(200, 96, dtype=torch.float64, generator=torch.Generator().manual_seed(8)).cuda()
    with torch.no_grad():
        a = build(False)(x)
        m = build(True)
        b1 = m(x)
        b2 = m(x)
    assert torch.equal(a, b1) and torch.equal(b1, b2)
