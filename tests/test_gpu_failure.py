"""Failure detection on the GPU without a GPU fault.

Every wait inside the GEMM is bounded.  These tests make one wait run out on
purpose and check what the caller sees, for both forms of the GEMM + CRT stage:
the library's test hook FPEMU_TEST_STALL_UNIT makes the TMA producers of the
kernel's first CTA pair stop delivering operand tiles (as a stalled producer
would); the MMA and epilogue warps of that pair then give up after
FPEMU_WAIT_BUDGET_MS (100 ms here), record FPEMU_ERR_TIMEOUT, mark what they
could not finish -- NaN over the fused kernel's output tile, an impossible
residue byte that the split form's CRT kernel turns into NaN -- and unwind,
while everything else is computed normally.  Nothing
traps and nothing faults; the context stays usable, which the second product
checks.  Each case runs in a fresh process because the wait budget is read
once per process.
"""
from __future__ import annotations

import os
import traceback

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

M, K, N = 1100, 700, 1300  # 5 x 6 tiles of 256 x 256, one tile per CTA pair


def _problem():
    rng = np.random.default_rng(5)
    A = (rng.random((M, K)) - 0.5) * np.exp(rng.standard_normal((M, K)))
    B = (rng.random((K, N)) - 0.5) * np.exp(rng.standard_normal((K, N)))
    return A, B


def _child(mode, path, q):
    try:
        os.environ["FPEMU_WAIT_BUDGET_MS"] = "100"
        os.environ["FPEMU_GEMM_PATH"] = path
        if mode == "sync":
            os.environ["FPEMU_CHECK"] = "1"
        else:
            os.environ.pop("FPEMU_CHECK", None)
        import torch

        from fp_emulation import _lib, ozaki2_int8_matmul

        dev = torch.device("cuda", 0)
        A, B = _problem()
        At, Bt = torch.from_numpy(A).to(dev), torch.from_numpy(B).to(dev)
        out = {}
        os.environ["FPEMU_TEST_STALL_UNIT"] = "1"  # the first pair stops after its first unit
        try:
            C = ozaki2_int8_matmul(At, Bt)
            torch.cuda.synchronize(dev)
            out["first_raised"] = None
            out["C"] = C.cpu().numpy()
            out["poll"] = _lib.poll_error()
        except _lib.FpemuError as exc:
            out["first_raised"] = (exc.status, str(exc))
        os.environ.pop("FPEMU_TEST_STALL_UNIT")
        try:
            C2 = ozaki2_int8_matmul(At, Bt)
            torch.cuda.synchronize(dev)
            out["second_raised"] = None
        except _lib.FpemuError as exc:
            out["second_raised"] = (exc.status, str(exc))
            C2 = ozaki2_int8_matmul(At, Bt)  # the error was cleared when it was raised
            torch.cuda.synchronize(dev)
        out["C2"] = C2.cpu().numpy()
        out["after"] = _lib.device_error(clear=True)
        q.put(("ok", out))
    except Exception:
        q.put(("error", traceback.format_exc()))


def _run(mode, path):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_child, args=(mode, path, q))
    p.start()
    status, out = q.get(timeout=240)
    p.join(timeout=60)
    assert status == "ok", out
    return out


def _check_partial(C, want, path):
    """Every output the stalled pair could not finish is NaN, every other one exact.
    Fused form: the first pair's tile, rows 0..255 x columns 0..255, is NaN.  Split
    form: the first pair's (tile, modulus) units after its first are spread over
    the product, and each tile with one of them unwritten is NaN."""
    nan = np.isnan(C)
    assert nan.any()
    if path == "fused":
        assert nan[:256, :256].all() and nan.sum() == 256 * 256
    np.testing.assert_array_equal(C[~nan].view(np.int64), want[~nan].view(np.int64))


PATHS = pytest.mark.parametrize("path", ["fused", "split"])


@PATHS
def test_timeout_raises_at_once_with_sync_checking(path):
    from fp_emulation import _lib
    from oracle import ozaki_oracle as oo

    out = _run("sync", path)
    assert out["first_raised"] is not None, "a timed-out product returned without an error"
    assert out["first_raised"][0] == _lib.FPEMU_ERR_TIMEOUT and "NaN" in out["first_raised"][1]
    assert out["second_raised"] is None
    A, B = _problem()
    np.testing.assert_array_equal(out["C2"].view(np.int64), oo.ozaki2_matmul(A, B).view(np.int64))
    assert out["after"][0] == 0


@PATHS
def test_timeout_shows_as_nan_and_raises_on_the_next_call_by_default(path):
    from fp_emulation import _lib
    from oracle import ozaki_oracle as oo

    out = _run("poll", path)
    A, B = _problem()
    want = oo.ozaki2_matmul(A, B)
    if out["first_raised"] is None:
        # The first call returned before its kernel finished: the tile it could
        # not finish is NaN, the host copy of the error record shows the timeout
        # without a synchronisation, and the next call raises.
        _check_partial(out["C"], want, path)
        code, where, _block, _detail = out["poll"]
        assert code == _lib.FPEMU_ERR_TIMEOUT and where in (1, 3), out["poll"]
        assert out["second_raised"] is not None and out["second_raised"][0] == _lib.FPEMU_ERR_TIMEOUT
    else:
        assert out["first_raised"][0] == _lib.FPEMU_ERR_TIMEOUT
    np.testing.assert_array_equal(out["C2"].view(np.int64), want.view(np.int64))
    assert out["after"][0] == 0
