"""Generate the golden fixtures by running the REFERENCE itself (CPU path).

Run in the build container, where the read-only reference tree exists:

    python tests/golden/make_golden.py

It imports thezettascale/fp-emulation from the reference source tree named by
``REF_SRC`` below (its CPU path JIT-builds ``crt_reconstruct.cpp``;
``LIBRARY_PATH`` gets gcc's libdir so ``-lgomp`` links, and the JIT cache goes
under ``oracle/_build/torch_ext``, git-ignored), runs the stage functions of
``ozaki.py`` on seeded inputs and saves inputs, every stage output and the
final result as ``tests/golden/*.npz``.  Large stage tensors are
stored as SHA-256 digests plus a few sampled planes to keep the fixtures small.

The fixtures pin the oracle (``oracle/ozaki_oracle.py``) to the reference
(``tests/test_oracle_golden.py``) and give the GPU tests known answers.
"""
from __future__ import annotations

import hashlib
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
# The reference's ``src`` directory (the parent of its fp_emulation package):
# FPEMU_REFERENCE_SRC names its fp_emulation directory, else the copy installed
# in baseline/_ref is used.
REF_SRC = (Path(os.environ["FPEMU_REFERENCE_SRC"]).parent if os.environ.get("FPEMU_REFERENCE_SRC")
           else REPO / "baseline" / "_ref")

# Stage tensors larger than this many elements are stored as digests + samples.
FULL_LIMIT = 40_000


def _setup_reference():
    sys.path.insert(0, str(REPO))
    from oracle.build_oracle import gcc_libdir

    os.environ["LIBRARY_PATH"] = gcc_libdir() + ":" + os.environ.get("LIBRARY_PATH", "")
    os.environ.setdefault("TORCH_EXTENSIONS_DIR", str(REPO / "oracle" / "_build" / "torch_ext"))
    sys.path.insert(0, str(REF_SRC))
    import fp_emulation.ozaki as oz  # the reference package

    assert Path(oz.__file__).resolve().is_relative_to(REF_SRC), oz.__file__
    return oz


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def wide(gen, n, m, phi, torch):
    """(U(0,1) - 0.5) * exp(phi * N(0,1)), the wide-dynamic-range inputs."""
    u = torch.rand(n, m, dtype=torch.float64, generator=gen)
    g = torch.randn(n, m, dtype=torch.float64, generator=gen)
    return (u - 0.5) * torch.exp(phi * g)


def cases(torch):
    """Yield (name, A, B) float tensors in the dtype the case runs in."""
    g = torch.Generator().manual_seed(0)  # config 1: 256x256 N(0,1), seed 0, A then B
    yield "cfg1_256", torch.randn(256, 256, dtype=torch.float64, generator=g), \
        torch.randn(256, 256, dtype=torch.float64, generator=g)

    g = torch.Generator().manual_seed(42)  # reference tests/test_ozaki.py:6-14
    yield "ref_accuracy_16", torch.randn(16, 16, dtype=torch.float64, generator=g), \
        torch.randn(16, 16, dtype=torch.float64, generator=g)

    g = torch.Generator().manual_seed(99)  # reference tests/test_ozaki.py:17-24
    yield "ref_rect_12x20x8", torch.randn(12, 20, dtype=torch.float64, generator=g), \
        torch.randn(20, 8, dtype=torch.float64, generator=g)

    # Odd shapes with an all-zero row and column, a row scaled by 2^40 and a
    # column scaled by 2^-40.
    g = torch.Generator().manual_seed(7)
    A = torch.randn(33, 70, dtype=torch.float64, generator=g)
    B = torch.randn(70, 45, dtype=torch.float64, generator=g)
    A[5] = 0.0
    B[:, 11] = 0.0
    A[9] *= 2.0 ** 40
    B[:, 3] *= 2.0 ** -40
    yield "odd_33x70x45_edges", A, B

    for phi in (0.5, 1.0, 2.0):  # config 2's wide-range distribution, small
        g = torch.Generator().manual_seed(1000 + int(phi * 10))
        yield f"wide_phi{phi}_64x96x80", wide(g, 64, 96, phi, torch), wide(g, 96, 80, phi, torch)

    # Config 3's distribution: N(0,1) with 1% of A's rows scaled by 2^40.
    g = torch.Generator().manual_seed(3)
    A = torch.randn(200, 128, dtype=torch.float64, generator=g)
    B = torch.randn(128, 72, dtype=torch.float64, generator=g)
    rows = torch.randperm(200, generator=g)[:2]
    A[rows] *= 2.0 ** 40
    yield "rows2p40_200x128x72", A, B

    # Extreme magnitudes: rows near 1e300 and 1e-300, subnormals, a column near 1e-200.
    g = torch.Generator().manual_seed(11)
    A = torch.randn(24, 40, dtype=torch.float64, generator=g)
    B = torch.randn(40, 20, dtype=torch.float64, generator=g)
    A[0] *= 1e300
    A[1] *= 1e-300
    A[2, :3] = torch.tensor([5e-324, -1e-310, 2.5e-320], dtype=torch.float64)
    A[2, 3:] = 0.0
    A[3, 7] = 1e-300 * 0.25  # a lone small value in an otherwise normal row
    B[:, 4] *= 1e-200
    yield "extremes_24x40x20", A, B

    # Inner dimension past the n_mod 24 -> 25 switch (k > 4096).
    g = torch.Generator().manual_seed(5)
    yield "k4100_6x4100x5", torch.randn(6, 4100, dtype=torch.float64, generator=g), \
        torch.randn(4100, 5, dtype=torch.float64, generator=g)

    # Exact ties for round-half-even: values that land on x.5 after scaling.
    A = torch.zeros(4, 8, dtype=torch.float64)
    A[:, 0] = 1.0  # row max 1 -> row_exp 1 -> scale 2^52
    A[0, 1:] = torch.tensor([2.0 ** -53, 3 * 2.0 ** -53, -(2.0 ** -53), -(3 * 2.0 ** -53),
                             5 * 2.0 ** -54, 2.0 ** -60, -0.5], dtype=torch.float64)
    A[1:, 1:] = torch.randn(3, 7, dtype=torch.float64, generator=torch.Generator().manual_seed(8))
    B = torch.randn(8, 6, dtype=torch.float64, generator=torch.Generator().manual_seed(9))
    yield "ties_4x8x6", A, B

    # Lower-precision dtypes (bits 24 / 11 / 8); the result is cast back.
    for dt in (torch.float32, torch.float16, torch.bfloat16):
        g = torch.Generator().manual_seed(21)
        A = torch.randn(40, 50, dtype=torch.float64, generator=g).to(dt)
        B = torch.randn(50, 30, dtype=torch.float64, generator=g).to(dt)
        yield f"dtype_{str(dt).split('.')[-1]}_40x50x30", A, B


def main():
    oz = _setup_reference()
    import torch

    HERE.mkdir(exist_ok=True)
    index = []
    for name, A, B in cases(torch):
        bits = oz._PRECISION_BITS[A.dtype]
        Ad, Bd = A.double(), B.double()
        n_mod = oz._n_moduli(Ad.shape[-1], bits)
        moduli = oz._PRIMES[:n_mod]
        A_int, B_int, row_exp, col_exp = oz._scale_to_int(Ad, Bd, bits)
        a_res = oz._residues(A_int, moduli)
        b_res = oz._residues(B_int, moduli)
        raw = (a_res.int() @ b_res.int())                       # ozaki.py:59 before the % p
        res = torch.stack(oz._matmul_residues(a_res, b_res, moduli))
        C = oz.ozaki2_int8_matmul(A, B)                         # the public op, dtype in = dtype out
        C64 = oz._reconstruct(list(res), moduli, bits, row_exp, col_exp)
        d = dict(
            A=Ad.numpy(), B=Bd.numpy(), bits=np.int32(bits), n_mod=np.int32(n_mod),
            dtype=np.bytes_(str(A.dtype).split(".")[-1]),
            row_exp=row_exp.numpy(), col_exp=col_exp.numpy(),
            A_int=A_int.numpy(), B_int=B_int.numpy(),
            C=C.double().numpy(), C64=C64.numpy(),
        )
        for key, t in (("a_res", a_res), ("b_res", b_res), ("raw", raw), ("res", res)):
            arr = t.numpy()
            d[f"{key}_sha256"] = np.bytes_(sha(arr))
            d[f"{key}_shape"] = np.asarray(arr.shape, dtype=np.int64)
            d[f"{key}_dtype"] = np.bytes_(str(arr.dtype))
            if arr.size <= FULL_LIMIT:
                d[key] = arr
            else:  # first and last modulus planes, full
                d[f"{key}_first"] = arr[0]
                d[f"{key}_last"] = arr[-1]
        if A.numel() + B.numel() > 2 * FULL_LIMIT:
            del d["A_int"], d["B_int"]
        np.savez_compressed(HERE / f"{name}.npz", **d)
        index.append(f"{name}: M={A.shape[0]} K={A.shape[1]} N={B.shape[1]} dtype={A.dtype} "
                     f"bits={bits} n_mod={n_mod}")
        print(index[-1])

    # Reference tests/test_nn.py:6-20: convert() of Linear(4,16)-Tanh-Linear(16,1), seed 42.
    from fp_emulation import convert  # the reference's nn.convert
    from torch import nn

    torch.manual_seed(42)
    model = nn.Sequential(nn.Linear(4, 16), nn.Tanh(), nn.Linear(16, 1))
    w = {k: v.detach().double().numpy().copy() for k, v in model.state_dict().items()}
    convert(model)
    x = torch.randn(2, 5, 4, dtype=torch.float64)
    y = model(x).detach()
    np.savez_compressed(HERE / "ref_convert_mlp.npz", x=x.numpy(), y=y.numpy(),
                        **{k.replace(".", "_"): v for k, v in w.items()})
    index.append("ref_convert_mlp: Sequential(Linear(4,16),Tanh,Linear(16,1)) seed 42, x [2,5,4]")

    # Backward: autograd through _OzakiMatmul (ozaki.py:132-136).
    g = torch.Generator().manual_seed(17)
    A = torch.randn(10, 14, dtype=torch.float64, generator=g, requires_grad=True)
    B = torch.randn(14, 6, dtype=torch.float64, generator=g, requires_grad=True)
    G = torch.randn(10, 6, dtype=torch.float64, generator=g)
    C = oz.ozaki2_int8_matmul(A, B)
    C.backward(G)
    np.savez_compressed(HERE / "ref_backward_10x14x6.npz", A=A.detach().numpy(),
                        B=B.detach().numpy(), G=G.numpy(), C=C.detach().numpy(),
                        dA=A.grad.numpy(), dB=B.grad.numpy())
    index.append("ref_backward_10x14x6: C = oz(A,B); C.backward(G); dA, dB")

    (HERE / "INDEX.txt").write_text(
        "Golden fixtures produced by running the reference's CPU path "
        "(tests/golden/make_golden.py).\n" + "\n".join(index) + "\n")


if __name__ == "__main__":
    main()
