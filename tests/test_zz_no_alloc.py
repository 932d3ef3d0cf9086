"""The allocation-free entry point, fpemu_gemm_crt_noalloc, through the C ABI.

Some callers cannot allocate device memory -- for example a host application
that owns the device allocator, or a runtime that forbids cudaMalloc between
launches.  For them the library offers a variant of the fused GEMM + CRT
stage that takes no workspace: its residue staging lives in a static 64 MiB
device array inside the library.  This test checks that variant against the
regular entry point (fpemu_gemm_crt, which stages in caller-provided
workspace) on two calls in a row with different problems, so the second call
runs over whatever the first left in the shared array.  Both must agree bit
for bit, the tolerance every parity test of this path uses, and a sampled
block of each result must equal the CPU oracle's.  A second test checks that
repeated calls leave the device's free memory exactly as it was.

The file is named to be collected last, and it needs nothing from the other
tests: it passes alone in a fresh process and after the rest of the suite.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _problem(seed, m, k, n):
    rng = np.random.default_rng(seed)
    A = (rng.random((m, k)) - 0.5) * np.exp(1.5 * rng.standard_normal((m, k)))
    B = (rng.random((k, n)) - 0.5) * np.exp(1.5 * rng.standard_normal((k, n)))
    return A, B


def _run_both(torch, lib, A_np, B_np):
    from fp_emulation import _lib
    from fp_emulation.ozaki import _n_moduli, _res_ld, _split

    dev = torch.device("cuda", 0)
    A = torch.from_numpy(A_np).to(dev)
    B = torch.from_numpy(B_np).to(dev)
    m, k = A.shape
    n = B.shape[1]
    n_mod = _n_moduli(k, 53)
    ld = _res_ld(k)
    a_res, re = _split(A, 53, n_mod)
    b_res, ce = _split(B.T, 53, n_mod)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)

    # Regular entry point: caller-provided workspace.
    C_ref = torch.full((m, n), float("nan"), dtype=torch.float64, device=dev)
    ws = torch.empty((lib.fpemu_gemm_workspace_size(m, n, n_mod),), dtype=torch.uint8, device=dev)
    _lib.check(lib.fpemu_gemm_crt(m, n, k, n_mod, a_res.data_ptr(), b_res.data_ptr(), ld, n * ld,
                                  re.data_ptr(), ce.data_ptr(), 53, C_ref.data_ptr(), n, 0, ws.data_ptr(),
                                  ws.numel(), stream),
               "fpemu_gemm_crt")

    # Allocation-free entry point: inputs and output only.
    C = torch.full((m, n), float("nan"), dtype=torch.float64, device=dev)
    _lib.check(lib.fpemu_gemm_crt_noalloc(m, n, k, n_mod, a_res.data_ptr(), b_res.data_ptr(), ld,
                                          re.data_ptr(), ce.data_ptr(), 53, C.data_ptr(), n, stream),
               "fpemu_gemm_crt_noalloc")
    torch.cuda.synchronize(dev)
    return C.cpu().numpy(), C_ref.cpu().numpy()


def test_noalloc_matches_regular_entry_point_twice():
    import torch

    from fp_emulation import _lib
    from oracle import ozaki_oracle as oo

    lib = _lib.load()
    # Two calls in a row: a larger problem (more tiles than the static area's
    # CTA budget, so the grid is the capped one), then a smaller one with a
    # different modulus count over the stale staging left by the first.
    for seed, (m, k, n) in ((1, (2304, 5000, 2600)), (2, (333, 700, 517))):
        A, B = _problem(seed, m, k, n)
        got, want = _run_both(torch, lib, A, B)
        assert not np.isnan(got).any()
        np.testing.assert_array_equal(got.view(np.int64), want.view(np.int64))
        # A block of rows x columns against the CPU oracle (exponents are per full
        # row of A and full column of B, so the block of the product is exact).
        rows = np.unique(np.r_[0, np.linspace(0, m - 1, 40).astype(int), m - 1])
        cols = np.unique(np.r_[0, np.linspace(0, n - 1, 60).astype(int), n - 1])
        block = oo.ozaki2_matmul(A[rows], B[:, cols])
        np.testing.assert_array_equal(got[np.ix_(rows, cols)].view(np.int64), block.view(np.int64))
    code = _lib.device_error(clear=True)
    assert code[0] == 0, f"device-side failure recorded: {code}"


def test_noalloc_leaves_free_device_memory_unchanged():
    """After a first call (which looks up the static array's address), further
    calls change the device's free memory by exactly zero bytes: nothing inside
    the library allocates, not even through an allocator torch cannot see."""
    import torch

    from fp_emulation import _lib
    from fp_emulation.ozaki import _n_moduli, _res_ld, _split

    lib = _lib.load()
    dev = torch.device("cuda", 0)
    A_np, B_np = _problem(3, 1000, 3000, 1200)
    A = torch.from_numpy(A_np).to(dev)
    B = torch.from_numpy(B_np).to(dev)
    m, k = A.shape
    n = B.shape[1]
    n_mod = _n_moduli(k, 53)
    ld = _res_ld(k)
    a_res, re = _split(A, 53, n_mod)
    b_res, ce = _split(B.T, 53, n_mod)
    C = torch.empty((m, n), dtype=torch.float64, device=dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)

    def call():
        _lib.check(lib.fpemu_gemm_crt_noalloc(m, n, k, n_mod, a_res.data_ptr(), b_res.data_ptr(), ld,
                                              re.data_ptr(), ce.data_ptr(), 53, C.data_ptr(), n, stream),
                   "fpemu_gemm_crt_noalloc")

    call()
    torch.cuda.synchronize(dev)
    free0, _ = torch.cuda.mem_get_info(dev)
    for _ in range(3):
        call()
    torch.cuda.synchronize(dev)
    free1, _ = torch.cuda.mem_get_info(dev)
    assert free1 == free0, f"free device memory changed by {free0 - free1} bytes"
    assert _lib.device_error(clear=True)[0] == 0
