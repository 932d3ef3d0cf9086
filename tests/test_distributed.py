"""Multi-rank host logic of the row-sharded product, on CPU ranks over gloo.

`fp_emulation.distributed.rowsharded_product` (chunked split + broadcast of B's
residues, split of the local rows of A, one fused GEMM per chunk) is run with
world_size 2 and a CPU backend built from the oracle, so the orchestration --
row shards, column chunks, who splits what, broadcast order, exponent
hand-off -- is checked bit for bit against the oracle's full product without a
GPU.  A second test makes one rank leave before the collectives and checks the
other fails within its process-group timeout instead of hanging.
"""
from __future__ import annotations

import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import ozaki_oracle as oo


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class OracleOps:
    """CPU stand-in for the GPU backend (tests only): same interface as _GpuOps."""

    def empty_res(self, n_mod, rows, ld):
        return torch.zeros((n_mod, rows, ld), dtype=torch.int8)

    def empty_exps(self, rows):
        return torch.zeros((rows,), dtype=torch.int32)

    def split(self, X, bits, n_mod, res, exps):
        Xn = X.contiguous().numpy()
        rows, k = Xn.shape
        A_int, _, re, _ = oo.scale_to_int(Xn, np.ones((k, 1)), bits)
        res.zero_()
        res[:, :, :k] = torch.from_numpy(oo.residues(A_int, oo.PRIMES[:n_mod]))
        exps.copy_(torch.from_numpy(re))

    def gemm_crt(self, a_res, re, b_res, ce_chunk, bits, C, c0, c1, k):
        n_mod = a_res.shape[0]
        moduli = oo.PRIMES[:n_mod]
        a = a_res[:, :, :k].numpy()
        b = b_res[:, :, :k].numpy().transpose(0, 2, 1)
        res = oo.matmul_residues(a, b, moduli)
        C[:, c0:c1] = torch.from_numpy(oo.reconstruct(res, moduli, bits, re.numpy(), ce_chunk.numpy()))


def _worker(rank, world, port, m, k, n, chunk_cols, out_q, drop_rank, mode="residues"):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.distributed.init_process_group("gloo", rank=rank, world_size=world,
                                             timeout=timedelta(seconds=4))
        from fp_emulation.distributed import rowsharded_product, shard_rows

        rng = np.random.default_rng(123)
        A = (rng.random((m, k)) - 0.5) * np.exp(rng.standard_normal((m, k)))
        B = (rng.random((k, n)) - 0.5) * np.exp(rng.standard_normal((k, n)))
        r0, r1 = shard_rows(m, world, rank)
        if rank == drop_rank:
            out_q.put((rank, "left", None))
            return  # leaves between steps, before any collective
        n_mod = oo.n_moduli(k, 53)
        C = rowsharded_product(torch.from_numpy(A[r0:r1]), torch.from_numpy(B) if rank == 0 else None,
                               n, k, 53, n_mod, OracleOps(), root=0, chunk_cols=chunk_cols, mode=mode)
        out_q.put((rank, "ok", (r0, r1, C.numpy())))
        torch.distributed.destroy_process_group()
    except Exception:
        out_q.put((rank, "error", traceback.format_exc()))


def _run(world, m, k, n, chunk_cols, drop_rank=-1, wait=120, mode="residues"):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, m, k, n, chunk_cols, q, drop_rank, mode))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=wait) for _ in range(world)]
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return results


@pytest.mark.parametrize("mode", ["residues", "fp64"])
@pytest.mark.parametrize("m,k,n,chunk", [(37, 90, 300, 256), (64, 300, 520, 512)])
def test_rowsharded_pipeline_matches_oracle(m, k, n, chunk, mode):
    results = _run(2, m, k, n, chunk, mode=mode)
    C = np.full((m, n), np.nan)
    for rank, status, payload in results:
        assert status == "ok", payload
        r0, r1, Cr = payload
        C[r0:r1] = Cr
    rng = np.random.default_rng(123)
    A = (rng.random((m, k)) - 0.5) * np.exp(rng.standard_normal((m, k)))
    B = (rng.random((k, n)) - 0.5) * np.exp(rng.standard_normal((k, n)))
    want = oo.ozaki2_matmul(A, B)
    np.testing.assert_array_equal(C.view(np.int64), want.view(np.int64))


def test_missing_rank_fails_instead_of_hanging():
    results = dict((r, (s, p)) for r, s, p in _run(2, 16, 40, 300, 256, drop_rank=1, wait=90))
    assert results[1][0] == "left"
    status, payload = results[0]
    assert status == "error", "rank 0 should fail when rank 1 never joins the broadcast"


def test_plan_column_chunks_and_shards():
    from fp_emulation.distributed import plan_column_chunks, shard_rows

    assert plan_column_chunks(1000, 256) == [(0, 256), (256, 512), (512, 768), (768, 1000)]
    assert plan_column_chunks(100, 2048) == [(0, 100)]
    assert plan_column_chunks(16384, 2048)[-1] == (14336, 16384)
    spans = [shard_rows(10, 4, r) for r in range(4)]
    assert spans == [(0, 3), (3, 6), (6, 8), (8, 10)]
