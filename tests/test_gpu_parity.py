"""GPU parity: every stage of the CUDA path against the oracle and the golden
fixtures produced by the reference, through the C ABI (via fp_emulation).

Bar: exponents, residues, raw int32 products and reduced residues bit-exact;
the final FP64 result bit-identical to the reference's CPU path (the CRT runs
the reference's operation order), which is stricter than the stated
"within 2 ulp" tolerance.
"""
from __future__ import annotations

import hashlib

import numpy as np
import pytest

from conftest import compensated_matmul, golden_names, load_golden, ulp_diff
from oracle import ozaki_oracle as oo

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["fused", "split"], autouse=True)
def gemm_path(request, monkeypatch):
    """Every test of this module runs on both forms of the GEMM + CRT stage: the
    fused kernel and the split form (spread residue GEMM, then the CRT kernel);
    FPEMU_GEMM_PATH forces one where the size would pick the other."""
    monkeypatch.setenv("FPEMU_GEMM_PATH", request.param)
    return request.param

ULP_TOL = 2  # north-star tolerance for the final FP64 result vs the reference


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    from fp_emulation import _lib

    _lib.load()
    yield torch
    code = _lib.device_error(clear=True)
    assert code[0] == 0, f"device-side failure recorded: {code}"


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _cuda(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _dtype(torch, g):
    return getattr(torch, g["dtype"].item().decode())


@pytest.mark.parametrize("split_rows", ["1", "2"], ids=["one-kernel", "two-kernel"])
@pytest.mark.parametrize("name", golden_names())
def test_split_stage_matches_reference(torch_cuda, name, split_rows, monkeypatch):
    """Both forms of the K-contiguous split (FPEMU_SPLIT_ROWS: the row maximum and
    the residues in one kernel, or in two) reproduce the reference's stages."""
    torch = torch_cuda
    from fp_emulation.ozaki import _split

    monkeypatch.setenv("FPEMU_SPLIT_ROWS", split_rows)
    g = load_golden(name)
    bits, n_mod = int(g["bits"]), int(g["n_mod"])
    A, B = _cuda(torch, g["A"]), _cuda(torch, g["B"])
    k = A.shape[1]
    a_res, re = _split(A, bits, n_mod)          # K contiguous
    b_res, ce = _split(B.T, bits, n_mod)        # K strided (B row-major)
    np.testing.assert_array_equal(re.cpu().numpy(), g["row_exp"])
    np.testing.assert_array_equal(ce.cpu().numpy(), g["col_exp"])
    a = a_res[:, :, :k].cpu().numpy()
    b = b_res[:, :, :k].cpu().numpy()
    assert np.all(a_res[:, :, k:].cpu().numpy() == 0) and np.all(b_res[:, :, k:].cpu().numpy() == 0)
    assert _sha(a) == g["a_res_sha256"].item().decode()
    assert _sha(np.ascontiguousarray(b.transpose(0, 2, 1))) == g["b_res_sha256"].item().decode()


@pytest.mark.parametrize("name", golden_names())
def test_gemm_stages_match_reference(torch_cuda, name):
    torch = torch_cuda
    from fp_emulation.ozaki import _matmul_residues, _reconstruct, _split

    g = load_golden(name)
    bits, n_mod = int(g["bits"]), int(g["n_mod"])
    A, B = _cuda(torch, g["A"]), _cuda(torch, g["B"])
    a_res, re = _split(A, bits, n_mod)
    b_res, ce = _split(B.T, bits, n_mod)
    raw = _matmul_residues(a_res, b_res, oo.PRIMES[:n_mod], raw=True).cpu().numpy()
    assert _sha(raw) == g["raw_sha256"].item().decode()
    res = _matmul_residues(a_res, b_res, oo.PRIMES[:n_mod]).cpu().numpy()
    assert _sha(res.astype(np.int32)) == g["res_sha256"].item().decode()
    C = _reconstruct(_cuda(torch, res), oo.PRIMES[:n_mod], bits, re, ce).cpu().numpy()
    np.testing.assert_array_equal(C.view(np.int64), g["C64"].view(np.int64))


@pytest.mark.parametrize("name", golden_names())
def test_end_to_end_matches_reference(torch_cuda, name):
    """The public op, fused path, bit-identical to the reference's CPU output
    (and therefore within ULP_TOL of it)."""
    torch = torch_cuda
    from fp_emulation import ozaki2_int8_matmul

    g = load_golden(name)
    dt = _dtype(torch, g)
    A = _cuda(torch, g["A"]).to(dt)
    B = _cuda(torch, g["B"]).to(dt)
    C = ozaki2_int8_matmul(A, B)
    assert C.dtype == dt
    got = C.double().cpu().numpy()
    assert np.max(ulp_diff(got, g["C"])) <= ULP_TOL
    np.testing.assert_array_equal(got.view(np.int64), g["C"].view(np.int64))


def test_reference_accuracy_case(torch_cuda):
    """Reference tests/test_ozaki.py:6-14 on the GPU: < 1e-14 from compensated."""
    torch = torch_cuda
    from fp_emulation import ozaki2_int8_matmul

    g = load_golden("ref_accuracy_16")
    C = ozaki2_int8_matmul(_cuda(torch, g["A"]), _cuda(torch, g["B"])).cpu().numpy()
    assert np.max(np.abs(C - compensated_matmul(g["A"], g["B"]))) < 1e-14


def test_reference_rect_case(torch_cuda):
    """Reference tests/test_ozaki.py:17-24: 12x20 @ 20x8, atol 1e-12 vs A @ B."""
    torch = torch_cuda
    from fp_emulation import ozaki2_int8_matmul

    gen = torch.Generator().manual_seed(99)
    A = torch.randn(12, 20, dtype=torch.float64, generator=gen)
    B = torch.randn(20, 8, dtype=torch.float64, generator=gen)
    C = ozaki2_int8_matmul(A.cuda(), B.cuda())
    assert C.shape == (12, 8)
    assert torch.allclose(C.cpu(), A @ B, atol=1e-12)


def test_reference_cuda_case(torch_cuda):
    """Reference tests/test_ozaki.py:27-35: CPU (reference output) vs CUDA, atol 1e-12."""
    torch = torch_cuda
    from fp_emulation import ozaki2_int8_matmul

    g = load_golden("ref_accuracy_16")
    C = ozaki2_int8_matmul(_cuda(torch, g["A"]), _cuda(torch, g["B"])).cpu()
    assert torch.allclose(torch.from_numpy(g["C"]), C, atol=1e-12)


def _rand_case(seed, m, k, n, kind="normal"):
    rng = np.random.default_rng(seed)
    if kind == "wide":
        A = (rng.random((m, k)) - 0.5) * np.exp(2.0 * rng.standard_normal((m, k)))
        B = (rng.random((k, n)) - 0.5) * np.exp(2.0 * rng.standard_normal((k, n)))
    else:
        A = rng.standard_normal((m, k))
        B = rng.standard_normal((k, n))
    return A, B


SHAPES = [(1, 1, 1), (1, 7, 1), (5, 1, 9), (127, 129, 255), (128, 128, 256), (129, 257, 257),
          (300, 1000, 77), (64, 4097, 40), (257, 300, 513)]


@pytest.mark.parametrize("m,k,n", SHAPES)
def test_odd_shapes_bit_exact_vs_oracle(torch_cuda, m, k, n):
    torch = torch_cuda
    from fp_emulation import ozaki2_int8_matmul

    A, B = _rand_case(m * 7919 + k * 31 + n, m, k, n, kind="wide" if (m + n) % 2 else "normal")
    want = oo.ozaki2_matmul(A, B)
    got = ozaki2_int8_matmul(_cuda(torch, A), _cuda(torch, B)).cpu().numpy()
    np.testing.assert_array_equal(got.view(np.int64), want.view(np.int64))


def test_k_at_the_int32_accumulation_limit(torch_cuda):
    """k = 214748, the largest inner dimension whose per-modulus int32 sums stay
    exact at n_mod = 25 (k * 100^2 < 2^31), is bit-exact against the oracle;
    one more is refused (the reference's int32 GEMM would overflow silently)."""
    torch = torch_cuda
    from fp_emulation import _lib, ozaki2_int8_matmul

    lib = _lib.load()
    kmax = lib.fpemu_max_k(25)
    assert kmax == 214748 and oo.n_moduli(kmax, 53) == 25
    rng = np.random.default_rng(5)
    A = (rng.random((3, kmax)) - 0.5) * np.exp(rng.standard_normal((3, kmax)))
    B = (rng.random((kmax, 2)) - 0.5) * np.exp(rng.standard_normal((kmax, 2)))
    A[:, :7] = 0.5  # residues near p-1 in many columns: large per-modulus sums
    want = oo.ozaki2_matmul(A, B)
    got = ozaki2_int8_matmul(_cuda(torch, A), _cuda(torch, B)).cpu().numpy()
    np.testing.assert_array_equal(got.view(np.int64), want.view(np.int64))
    with pytest.raises(_lib.FpemuError, match="int32"):
        ozaki2_int8_matmul(torch.ones(2, kmax + 1, dtype=torch.float64, device="cuda"),
                           torch.ones(kmax + 1, 2, dtype=torch.float64, device="cuda"))


def test_transposed_and_strided_views(torch_cuda):
    """A and B given as transposed / sliced views: no copies, same bits."""
    torch = torch_cuda
    from fp_emulation import ozaki2_int8_matmul

    A, B = _rand_case(3, 150, 200, 90)
    want = oo.ozaki2_matmul(A, B)
    At = _cuda(torch, A.T.copy()).T            # A as a transposed view (K strided)
    Bt = _cuda(torch, B.T.copy()).T            # B as a transposed view (K contiguous)
    for a, b in [(At, _cuda(torch, B)), (_cuda(torch, A), Bt), (At, Bt)]:
        got = ozaki2_int8_matmul(a, b).cpu().numpy()
        np.testing.assert_array_equal(got.view(np.int64), want.view(np.int64))
    big = _cuda(torch, np.pad(A, ((0, 0), (3, 5))))[:, 3:203]  # row stride 208, offset 3
    got = ozaki2_int8_matmul(big, _cuda(torch, B)).cpu().numpy()
    np.testing.assert_array_equal(got.view(np.int64), want.view(np.int64))


@pytest.mark.parametrize("n", [512, 1024])
def test_medium_square_bit_exact_vs_oracle(torch_cuda, n):
    torch = torch_cuda
    from fp_emulation import ozaki2_int8_matmul

    A, B = _rand_case(n, n, n, n, kind="wide")
    want = oo.ozaki2_matmul(A, B)
    got = ozaki2_int8_matmul(_cuda(torch, A), _cuda(torch, B)).cpu().numpy()
    np.testing.assert_array_equal(got.view(np.int64), want.view(np.int64))


def test_modulus_sweep(torch_cuda):
    """n_mod below the reference default (config 2's sweep): same bits as the
    oracle with that modulus count, and the error shrinks as n_mod grows."""
    torch = torch_cuda
    from fp_emulation.ozaki import _ozaki2_forward

    A, B = _rand_case(11, 96, 256, 80)
    exact = A @ B
    errs = []
    for n_mod in (16, 20, 22, 24):
        want = oo.ozaki2_matmul(A, B, n_mod=n_mod)
        got = _ozaki2_forward(_cuda(torch, A), _cuda(torch, B), n_mod=n_mod).cpu().numpy()
        np.testing.assert_array_equal(got.view(np.int64), want.view(np.int64))
        errs.append(np.max(np.abs(got - exact)))
    assert errs[-1] < 1e-12 and errs[0] > errs[-1]


def test_convert_mlp_matches_reference(torch_cuda):
    """Reference tests/test_nn.py:6-20 (golden output of the reference's convert())."""
    torch = torch_cuda
    from torch import nn

    from fp_emulation import convert

    g = load_golden("ref_convert_mlp")
    model = nn.Sequential(nn.Linear(4, 16), nn.Tanh(), nn.Linear(16, 1))
    with torch.no_grad():
        for i in (0, 2):
            model[i].weight.copy_(torch.from_numpy(g[f"{i}_weight"]))
            model[i].bias.copy_(torch.from_numpy(g[f"{i}_bias"]))
    convert(model)
    model = model.cuda()
    x = _cuda(torch, g["x"])
    y = model(x).detach().cpu().numpy()
    # The reference's own tolerance (test_nn.py:20); torch.tanh on CUDA and on
    # the CPU differ in the last bits, so the whole network is not bit-exact.
    np.testing.assert_allclose(y, g["y"], rtol=0, atol=1e-12)
    assert model[0].weight.dtype == torch.float64
    # Each emulated Linear on its own input is bit-exact vs the oracle.
    h = x.reshape(-1, 4)
    with torch.no_grad():
        for layer in (model[0], model[2]):
            got = layer(h).cpu().numpy()
            want = oo.ozaki2_matmul(h.cpu().numpy(), layer.weight.cpu().numpy().T) + layer.bias.cpu().numpy()
            np.testing.assert_array_equal(got.view(np.int64), want.view(np.int64))
            h = torch.tanh(layer(h))


def test_backward_matches_reference(torch_cuda):
    torch = torch_cuda
    from fp_emulation import ozaki2_int8_matmul

    g = load_golden("ref_backward_10x14x6")
    A = _cuda(torch, g["A"]).requires_grad_(True)
    B = _cuda(torch, g["B"]).requires_grad_(True)
    C = ozaki2_int8_matmul(A, B)
    C.backward(_cuda(torch, g["G"]))
    for got, want in ((C.detach(), g["C"]), (A.grad, g["dA"]), (B.grad, g["dB"])):
        np.testing.assert_array_equal(got.cpu().numpy().view(np.int64), want.view(np.int64))


def test_nonfinite_rows_give_nan(torch_cuda):
    """NaN/Inf are outside the reference's contract; this build defines them:
    a row of A (column of B) holding NaN or Inf makes that output row (column) NaN."""
    torch = torch_cuda
    from fp_emulation import ozaki2_int8_matmul

    A, B = _rand_case(5, 8, 16, 6)
    A[2, 3] = np.nan
    B[4, 1] = np.inf
    C = ozaki2_int8_matmul(_cuda(torch, A), _cuda(torch, B)).cpu().numpy()
    assert np.all(np.isnan(C[2])) and np.all(np.isnan(C[:, 1]))
    mask = np.ones_like(C, dtype=bool)
    mask[2] = False
    mask[:, 1] = False
    A[2, 3] = 0.0
    B[4, 1] = 0.0
    want = oo.ozaki2_matmul(A, B)
    np.testing.assert_array_equal(C[mask], want[mask])


@pytest.mark.parametrize("sched", ["modulus", "modulus-tail", "tile"])
@pytest.mark.parametrize("ctas", ["1", "2"])
@pytest.mark.parametrize("m,k,n", [(300, 520, 700), (513, 1100, 257), (1000, 300, 1000), (2600, 200, 700)])
def test_gemm_configurations_agree(torch_cuda, monkeypatch, sched, ctas, m, k, n):
    """The CTA-pair GEMM (default) and the single-CTA GEMM (FPEMU_GEMM_CTAS=1),
    each with the modulus-major schedule (default; "modulus-tail": the last
    two passes interleaved, FPEMU_GEMM_TAIL=1) and the tile-major one
    (FPEMU_GEMM_SCHED=tile), must reproduce the oracle bit for bit, in the
    fused mode and in both parity taps."""
    torch = torch_cuda
    from fp_emulation import ozaki2_int8_matmul
    from fp_emulation.ozaki import _matmul_residues, _split

    monkeypatch.setenv("FPEMU_GEMM_CTAS", ctas)
    monkeypatch.setenv("FPEMU_GEMM_SCHED", "tile" if sched == "tile" else "modulus")
    monkeypatch.setenv("FPEMU_GEMM_TAIL", "1" if sched == "modulus-tail" else "0")
    A, B = _rand_case(m + k + n, m, k, n, kind="wide")
    C, st = oo.ozaki2_matmul(A, B, stages=True)
    got = ozaki2_int8_matmul(_cuda(torch, A), _cuda(torch, B)).cpu().numpy()
    np.testing.assert_array_equal(got.view(np.int64), C.view(np.int64))
    a_res, _ = _split(_cuda(torch, A), 53, len(st["moduli"]))
    b_res, _ = _split(_cuda(torch, B).T, 53, len(st["moduli"]))
    raw = _matmul_residues(a_res, b_res, st["moduli"], raw=True).cpu().numpy()
    np.testing.assert_array_equal(raw, oo.matmul_residues_raw(st["a_res"], st["b_res"]).astype(np.int32))
    res = _matmul_residues(a_res, b_res, st["moduli"]).cpu().numpy()
    np.testing.assert_array_equal(res.astype(np.int32), st["res"])
