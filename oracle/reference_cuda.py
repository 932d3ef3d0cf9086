"""The reference's own CUDA path, timed on the GPU.  BENCH INFRASTRUCTURE ONLY.

``bench.py --sweep`` runs this module as a child process,
``python -m oracle.reference_cuda '<json list of points>'``, because the
reference package and this repository's drop-in are both named
``fp_emulation``.  The child imports the unmodified reference package
installed in ``baseline/_ref``, gives its ``_cuda_crt`` loader
(``_cuda_crt.py:11-21``) the extension that ``oracle/build_oracle.py`` compiled
from the reference's ``crt_kernel.cu`` -- what the reference's JIT build
produces -- and times ``ozaki2_int8_matmul(A, B)`` on CUDA tensors with CUDA
events: the reference's torch scaling and residue steps (ozaki.py:32-46),
its cuBLASLt strided-batched INT8 GEMM and ``mod_reduce``, and its
``crt_kernel`` (crt_kernel.cu:6-146).  Points where the reference's int32
element indices would overflow (n_mod * m * n >= 2^31, crt_kernel.cu:87-108)
are skipped, not run.

Inputs are generated exactly as bench.py generates its own (same seeded
torch generator calls on the same device), so the parent can compare a block
of the two results.  Output: one JSON line, a list of per-point records.
"""
from __future__ import annotations

import importlib.util
import json
import math
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent


def synth(torch, rows, cols, phi, seed, device):
    """bench.py's config-2 inputs: (U(0,1) - 0.5) * exp(phi * N(0,1)), seeded."""
    g = torch.Generator(device=device).manual_seed(seed)
    u = torch.rand(rows, cols, dtype=torch.float64, generator=g, device=device)
    e = torch.randn(rows, cols, dtype=torch.float64, generator=g, device=device)
    return (u - 0.5) * torch.exp(phi * e)


def main(points):
    sys.path = [p for p in sys.path if not p.rstrip("/").endswith("fp-emulation_b200")]
    ref_root = REPO / "baseline" / "_ref"
    sys.path.insert(0, str(ref_root))
    import torch

    import fp_emulation
    import fp_emulation._cuda_crt as cc
    from fp_emulation.ozaki import _n_moduli

    assert Path(fp_emulation.__file__).resolve().is_relative_to(ref_root.resolve()), fp_emulation.__file__
    sys.path.insert(1, str(REPO))
    from oracle.build_oracle import build_ref_cuda, ref_cuda_module_path

    so = ref_cuda_module_path() or build_ref_cuda()
    spec = importlib.util.spec_from_file_location("crt_cuda_ref", str(so))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    cc._module = mod  # what cc._load() would return after its JIT build

    dev = torch.device("cuda", 0)
    out = []
    for pt in points:
        n, phi = pt["n"], pt["phi"]
        n_mod = _n_moduli(n, 53)
        rec = {"n": n, "phi": phi, "n_mod": n_mod}
        if n_mod * n * n >= 2 ** 31:
            rec["skipped"] = "n_mod*m*n >= 2^31 overflows the reference's int32 element indices"
            out.append(rec)
            continue
        A = synth(torch, n, n, phi, pt["seed_a"], dev)
        B = synth(torch, n, n, phi, pt["seed_b"], dev)
        for _ in range(pt["warmup"]):
            fp_emulation.ozaki2_int8_matmul(A, B)
        torch.cuda.synchronize(dev)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(pt["steps"]):
            C = fp_emulation.ozaki2_int8_matmul(A, B)
        e.record()
        torch.cuda.synchronize(dev)
        ms = s.elapsed_time(e) / pt["steps"]
        blk = C[: pt["block"], : pt["block"]].cpu().flatten().tolist()
        rec.update(ms=round(ms, 4), tflops=round(2.0 * n ** 3 / (ms * 1e-3) / 1e12, 4),
                   block=[float.hex(v) for v in blk])
        del A, B, C
        torch.cuda.empty_cache()
        out.append(rec)
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main(json.loads(sys.argv[1]))
