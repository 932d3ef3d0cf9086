"""The public op inside a CUDA graph.  Launch-bound callers (small products in
a training step) capture the library's calls: after one eager call on the
device (which sets up the per-device state -- error watch, occupancy, kernel
attributes), a product is captured once and replayed on new inputs written into
the same buffers, and every replay must give the oracle's result bit for bit,
for both forms of the GEMM + CRT stage."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import ozaki_oracle as oo

pytestmark = pytest.mark.gpu


def _inputs(seed, m, k, n):
    rng = np.random.default_rng(seed)
    A = (rng.random((m, k)) - 0.5) * np.exp(rng.standard_normal((m, k)))
    B = (rng.random((k, n)) - 0.5) * np.exp(rng.standard_normal((k, n)))
    return A, B


@pytest.mark.parametrize("path", ["fused", "split"])
def test_product_captured_in_a_cuda_graph_replays_exactly(path, monkeypatch):
    import torch

    from fp_emulation import _lib, ozaki2_int8_matmul

    monkeypatch.setenv("FPEMU_GEMM_PATH", path)
    dev = torch.device("cuda", 0)
    m, k, n = 300, 520, 410
    A0, B0 = _inputs(1, m, k, n)
    A = torch.from_numpy(A0).to(dev)
    B = torch.from_numpy(B0).to(dev)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        ozaki2_int8_matmul(A, B)  # eager first call: per-device set-up
    torch.cuda.current_stream(dev).wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        C = ozaki2_int8_matmul(A, B)
    for seed in (2, 3):
        An, Bn = _inputs(seed, m, k, n)
        A.copy_(torch.from_numpy(An))
        B.copy_(torch.from_numpy(Bn))
        g.replay()
        torch.cuda.synchronize(dev)
        np.testing.assert_array_equal(C.cpu().numpy().view(np.int64), oo.ozaki2_matmul(An, Bn).view(np.int64))
    assert _lib.device_error(clear=True)[0] == 0
