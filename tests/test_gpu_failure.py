"""Failure detection on the GPU without a GPU fault.

Every wait inside the fused GEMM is bounded.  These tests make one wait run
out on purpose and check what the caller sees: the library's test hook
FPEMU_TEST_STALL_UNIT makes the TMA producers of the kernel's first CTA pair
stop delivering operand tiles (as a stalled producer would); the MMA and
epilogue warps of that pair then give up after FPEMU_WAIT_BUDGET_MS (100 ms
here), record FPEMU_ERR_TIMEOUT, write NaN over the output tile they could not
finish and unwind, while every other tile is computed normally.  Nothing
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


def _child(mode, q):
    try:
        os.environ["FPEMU_WAIT_BUDGET_MS"] = "100"
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


def _run(mode):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_child, args=(mode, q))
    p.start()
    status, out = q.get(timeout=240)
    p.join(timeout=60)
    assert status == "ok", out
    return out


def _check_partial(C, want):
    # The first pair's tile is rows 0..255, columns 0..255 of C: NaN; the rest exact.
    assert np.isnan(C[:256, :256]).all()
    rest = np.ones(C.shape, dtype=bool)
    rest[:256, :256] = False
    np.testing.assert_array_equal(C[rest].view(np.int64), want[rest].view(np.int64))


def test_timeout_raises_at_once_with_sync_checking():
    from fp_emulation import _lib
    from oracle import ozaki_oracle as oo

    out = _run("sync")
    assert out["first_raised"] is not None, "a timed-out product returned without an error"
    assert out["first_raised"][0] == _lib.FPEMU_ERR_TIMEOUT and "NaN" in out["first_raised"][1]
    assert out["second_raised"] is None
    A, B = _problem()
    np.testing.assert_array_equal(out["C2"].view(np.int64), oo.ozaki2_matmul(A, B).view(np.int64))
    assert out["after"][0] == 0


def test_timeout_shows_as_nan_and_raises_on_the_next_call_by_default():
    from fp_emulation import _lib
    from oracle import ozaki_oracle as oo

    out = _run("poll")
    A, B = _problem()
    want = oo.ozaki2_matmul(A, B)
    if out["first_raised"] is None:
        # The first call returned before its kernel finished: the tile it could
        # not finish is NaN, the host copy of the error record shows the timeout
        # without a synchronisation, and the next call raises.
        _check_partial(out["C"], want)
        code, where, _block, _detail = out["poll"]
        assert code == _lib.FPEMU_ERR_TIMEOUT and where in (1, 3), out["poll"]
        assert out["second_raised"] is not None and out["second_raised"][0] == _lib.FPEMU_ERR_TIMEOUT
    else:
        assert out["first_raised"][0] == _lib.FPEMU_ERR_TIMEOUT
    np.testing.assert_array_equal(out["C2"].view(np.int64), want.view(np.int64))
    assert out["after"][0] == 0
