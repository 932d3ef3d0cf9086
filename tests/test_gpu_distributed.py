"""The row-sharded multi-GPU product on real GPUs: 2 NCCL ranks as child
processes (skipped with fewer than 2 GPUs).  Each rank computes its rows of C
through the pipelined broadcast of B's residues; the gathered result must be
bit-identical to the oracle's full product."""
from __future__ import annotations

import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest

from oracle import ozaki_oracle as oo

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem(m, k, n):
    rng = np.random.default_rng(77)
    A = (rng.random((m, k)) - 0.5) * np.exp(1.5 * rng.standard_normal((m, k)))
    B = (rng.random((k, n)) - 0.5) * np.exp(1.5 * rng.standard_normal((k, n)))
    return A, B


def _worker(rank, world, port, m, k, n, q, transport="ce", calls=2):
    try:
        import torch

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                          FPEMU_CHUNK_COLS="512", FPEMU_TRANSPORT=transport)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        torch.distributed.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                             timeout=timedelta(seconds=60))
        from fp_emulation import _lib
        from fp_emulation.distributed import ozaki2_int8_matmul_rowsharded, shard_rows

        A, B = _problem(m, k, n)
        r0, r1 = shard_rows(m, world, rank)
        A_local = torch.from_numpy(A[r0:r1]).to(dev)
        B_t = torch.from_numpy(B).to(dev) if rank == 0 else None
        # Several calls in a row: buffers and events of the transport are reused.
        for _ in range(calls):
            C = ozaki2_int8_matmul_rowsharded(A_local, B_t, n=n, root=0)
        torch.cuda.synchronize(dev)
        code = _lib.device_error(clear=True)
        q.put((rank, "ok", (r0, r1, C.cpu().numpy(), code)))
        torch.distributed.barrier(device_ids=[rank])
        torch.distributed.destroy_process_group()
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


@pytest.mark.parametrize("transport", ["ce", "nccl"])
def test_rowsharded_two_gpus_bit_exact(transport):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    m, k, n = 1000, 700, 1500
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, m, k, n, q, transport)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    C = np.full((m, n), np.nan)
    for rank, status, payload in results:
        assert status == "ok", payload
        r0, r1, Cr, code = payload
        assert code[0] == 0, code
        C[r0:r1] = Cr
    A, B = _problem(m, k, n)
    np.testing.assert_array_equal(C.view(np.int64), oo.ozaki2_matmul(A, B).view(np.int64))
