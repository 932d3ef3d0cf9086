"""The reference-side binding on a GPU.

1. ``fpemu_ozaki2_dgemm`` -- the one-shot entry point the reference's binding
   calls -- through ctypes, bit-identical to the reference's own CPU output
   (golden fixtures made by running the reference) for contiguous and strided
   operands.
2. The unmodified reference package, installed in ``baseline/_ref``, with the
   binding stub ``fp-emulation_b200/reference_binding/_fpemu.py`` added as
   ``fp_emulation._fpemu`` and the three-line CUDA branch inserted into its
   ``_ozaki2_forward`` after ``moduli = _PRIMES[:n_mod]`` (ozaki.py:109):
   ``ozaki2_int8_matmul(A.cuda(), B.cuda())`` through the reference's own API
   must equal the reference's CPU output bit for bit -- the reference's
   test_cuda (tests/test_ozaki.py:27-35, atol 1e-12) with the stricter bar.
   Runs in a child process so that the reference's ``fp_emulation`` does not
   meet this repository's package of the same name.
"""
from __future__ import annotations

import ctypes
import json
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

from conftest import REPO, load_golden

pytestmark = pytest.mark.gpu

REF_PKG = REPO / "baseline" / "_ref"
STUB = REPO / "fp-emulation_b200" / "reference_binding" / "_fpemu.py"
LIB = REPO / "fp-emulation_b200" / "fp_emulation" / "libfpemu.so"


@pytest.mark.parametrize("case", ["cfg1_256", "ref_rect_12x20x8", "odd_33x70x45_edges"])
@pytest.mark.parametrize("layout", ["contiguous", "transposed"])
def test_one_shot_entry_point_matches_reference_golden(case, layout):
    import torch

    from fp_emulation import _lib

    g = load_golden(case)
    A_np, B_np, want = g["A"], g["B"], g["C"]
    dev = torch.device("cuda", 0)
    if layout == "contiguous":
        A = torch.from_numpy(A_np).to(dev)
        B = torch.from_numpy(B_np).to(dev)
    else:  # both operands as transposed views of column-major storage
        A = torch.from_numpy(np.ascontiguousarray(A_np.T)).to(dev).T
        B = torch.from_numpy(np.ascontiguousarray(B_np.T)).to(dev).T
    m, k = A.shape
    n = B.shape[1]
    lib = _lib.load()
    n_mod = ctypes.c_int(0)
    _lib.check(lib.fpemu_plan_moduli(k, 53, ctypes.byref(n_mod), None))
    ws = torch.empty((lib.fpemu_workspace_size(m, n, k, n_mod.value),), dtype=torch.uint8, device=dev)
    C = torch.full((m, n), float("nan"), dtype=torch.float64, device=dev)
    st = lib.fpemu_ozaki2_dgemm(m, n, k, A.data_ptr(), A.stride(0), A.stride(1), B.data_ptr(), B.stride(0),
                                B.stride(1), C.data_ptr(), n, 53, 0, ws.data_ptr(), ws.numel(),
                                ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    _lib.check(st, "fpemu_ozaki2_dgemm")
    got = C.cpu().numpy()
    np.testing.assert_array_equal(got.view(np.int64), want.view(np.int64))


_CHILD = textwrap.dedent('''
    import importlib.util, inspect, json, sys
    import numpy as np
    sys.path.insert(0, REF_PKG)
    import torch
    import fp_emulation as ref
    import fp_emulation.ozaki as ro
    assert ref.__file__.startswith(REF_PKG), ref.__file__
    spec = importlib.util.spec_from_file_location("fp_emulation._fpemu", STUB)
    stub = importlib.util.module_from_spec(spec)
    sys.modules["fp_emulation._fpemu"] = stub
    spec.loader.exec_module(stub)
    # Insert the binding's CUDA branch into the reference's _ozaki2_forward.
    src = inspect.getsource(ro._ozaki2_forward)
    anchor = "    moduli = _PRIMES[:n_mod]\\n"
    assert anchor in src
    branch = ("    if A.is_cuda:\\n"
              "        from fp_emulation._fpemu import cuda_ozaki2\\n"
              "        result = cuda_ozaki2(A, B, bits, n_mod)\\n"
              "        return result if orig_dtype == torch.float64 else result.to(orig_dtype)\\n")
    exec(src.replace(anchor, anchor + branch), ro.__dict__)
    out = {}
    for name in CASES:
        z = np.load(name)
        A, B, want = z["A"], z["B"], z["C"]
        C = ref.ozaki2_int8_matmul(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()).cpu().numpy()
        out[name] = bool(np.array_equal(C.view(np.int64), want.view(np.int64)))
    # Autograd through the reference's own _OzakiMatmul: backward re-enters the binding.
    z = np.load(BACKWARD)
    A = torch.from_numpy(z["A"]).cuda().requires_grad_(True)
    B = torch.from_numpy(z["B"]).cuda().requires_grad_(True)
    C = ref.ozaki2_int8_matmul(A, B)
    C.backward(torch.from_numpy(z["G"]).cuda())
    out["backward"] = bool(np.array_equal(A.grad.cpu().numpy().view(np.int64), z["dA"].view(np.int64)) and
                           np.array_equal(B.grad.cpu().numpy().view(np.int64), z["dB"].view(np.int64)))
    print(json.dumps(out))
''')


def test_reference_package_with_the_binding_stub():
    if not (REF_PKG / "fp_emulation" / "ozaki.py").exists():
        pytest.skip("the reference package is not installed in baseline/_ref")
    cases = [str(REPO / "tests" / "golden" / f"{c}.npz") for c in ("ref_accuracy_16", "cfg1_256", "ref_rect_12x20x8")]
    back = REPO / "tests" / "golden" / "ref_backward_10x14x6.npz"
    code = (f"REF_PKG = {str(REF_PKG)!r}\nSTUB = {str(STUB)!r}\nCASES = {cases!r}\nBACKWARD = {str(back)!r}\n"
            + _CHILD)
    env = dict(os.environ, FPEMU_LIB=str(LIB))
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=600,
                         cwd="/")
    assert res.returncode == 0, res.stdout + res.stderr
    out = json.loads(res.stdout.strip().splitlines()[-1])
    assert all(out.values()), out
