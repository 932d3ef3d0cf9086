"""The segmented epilogue (fpemu_gemm_crt_segmented) on one GPU: a product
over columns gathered from several column blocks of C writes each column to
its place.  B = [block 0 | block 1 | block 2] (90 columns each); the product
over strip [30, 60) of every block -- the shape of one chunk of the
column-sharded multi-GPU product -- must fill exactly those columns of C, bit
for bit equal to the oracle, and leave every other column untouched."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import ozaki_oracle as oo

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("path", ["fused", "split"])
def test_segmented_columns_land_in_their_blocks(path, monkeypatch):
    import torch

    monkeypatch.setenv("FPEMU_GEMM_PATH", path)
    from fp_emulation import _lib
    from fp_emulation.ozaki import _n_moduli, _res_ld, _split

    rng = np.random.default_rng(21)
    m, k, nb, W, s0, s1 = 150, 333, 90, 3, 30, 60
    A = (rng.random((m, k)) - 0.5) * np.exp(rng.standard_normal((m, k)))
    B = (rng.random((k, W * nb)) - 0.5) * np.exp(rng.standard_normal((k, W * nb)))
    cols = np.concatenate([q * nb + np.arange(s0, s1) for q in range(W)])
    dev = torch.device("cuda", 0)
    n_mod = _n_moduli(k, 53)
    a_res, re = _split(torch.from_numpy(A).to(dev), 53, n_mod)
    b_res, ce = _split(torch.from_numpy(B[:, cols]).to(dev).T, 53, n_mod)  # the gathered chunk
    C = torch.full((m, W * nb), 7.0, dtype=torch.float64, device=dev)
    lib = _lib.load()
    w = len(cols)
    ws = torch.empty((lib.fpemu_gemm_workspace_size(m, w, n_mod),), dtype=torch.uint8, device=dev)
    st = lib.fpemu_gemm_crt_segmented(m, w, k, n_mod, a_res.data_ptr(), b_res.data_ptr(), _res_ld(k),
                                      b_res.stride(0), re.data_ptr(), ce.data_ptr(), 53, C.data_ptr() + 8 * s0,
                                      W * nb, s1 - s0, nb, 0, ws.data_ptr(), ws.numel(),
                                      ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    _lib.check(st, "fpemu_gemm_crt_segmented")
    got = C.cpu().numpy()
    want = oo.ozaki2_matmul(A, B[:, cols])
    np.testing.assert_array_equal(got[:, cols].view(np.int64), want.view(np.int64))
    rest = np.setdiff1d(np.arange(W * nb), cols)
    assert (got[:, rest] == 7.0).all()
    # A segment layout whose last column would land past the row is refused.
    st = lib.fpemu_gemm_crt_segmented(m, w, k, n_mod, a_res.data_ptr(), b_res.data_ptr(), _res_ld(k),
                                      b_res.stride(0), re.data_ptr(), ce.data_ptr(), 53, C.data_ptr(),
                                      W * nb, s1 - s0, 2 * nb, 0, ws.data_ptr(), ws.numel(), None)
    assert st == _lib.FPEMU_ERR_INVALID
