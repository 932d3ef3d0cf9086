"""The row-sharded multi-GPU product on real GPUs: NCCL ranks as child
processes (skipped with too few GPUs).  Each rank computes its rows of C
through the pipelined broadcast of B's residues; the gathered result must be
bit-identical to the oracle's full product."""
from __future__ import annotations

import os
import traceback
from datetime import timedelta

import numpy as np
import pytest

from oracle import ozaki_oracle as oo

pytestmark = pytest.mark.gpu


def _problem(m, k, n):
    rng = np.random.default_rng(77)
    A = (rng.random((m, k)) - 0.5) * np.exp(1.5 * rng.standard_normal((m, k)))
    B = (rng.random((k, n)) - 0.5) * np.exp(1.5 * rng.standard_normal((k, n)))
    return A, B


def _worker(rank, world, store_file, m, k, n, q, transport="ce", calls=2):
    try:
        import torch

        os.environ.update(NCCL_NVLS_ENABLE="0", FPEMU_CHUNK_COLS="512", FPEMU_TRANSPORT=transport)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        # A file store: no TCP port to collide with an earlier test's sockets.
        torch.distributed.init_process_group("nccl", init_method=f"file://{store_file}", rank=rank,
                                             world_size=world, device_id=dev, timeout=timedelta(seconds=60))
        from fp_emulation import _lib
        from fp_emulation.distributed import ozaki2_int8_matmul_rowsharded, shard_rows

        A, B = _problem(m, k, n)
        r0, r1 = shard_rows(m, world, rank)
        A_local = torch.from_numpy(A[r0:r1]).to(dev)
        B_t = torch.from_numpy(B).to(dev) if rank == 0 else None
        # Several calls in a row: buffers and events of the transport are reused.
        for _ in range(calls):
            C = ozaki2_int8_matmul_rowsharded(A_local, B_t, n=n, root=0)
        # A second column count in the same group: a second transport channel,
        # whose handshakes must not be confused with the first one's.
        n2 = n // 2 + 1
        C2 = ozaki2_int8_matmul_rowsharded(A_local, B_t[:, :n2].contiguous() if B_t is not None else None,
                                           n=n2, root=0)
        C = ozaki2_int8_matmul_rowsharded(A_local, B_t, n=n, root=0)
        torch.cuda.synchronize(dev)
        code = _lib.device_error(clear=True)
        q.put((rank, "ok", (r0, r1, C.cpu().numpy(), C2.cpu().numpy(), code)))
        torch.distributed.barrier(device_ids=[rank])
        torch.distributed.destroy_process_group()
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


@pytest.mark.parametrize("world", [2, "all"])
@pytest.mark.parametrize("transport", ["ce", "ce-ring", "nccl"])
def test_rowsharded_multi_gpu_bit_exact(transport, world, tmp_path):
    """world 2: root and last rank only; "all" (3 or more GPUs): the chain's middle
    ranks both receive from a predecessor and feed a successor."""
    import torch
    import torch.multiprocessing as mp

    have = torch.cuda.device_count()
    if world == "all":
        if have < 3:
            pytest.skip("needs 3 or more GPUs")
        world = have
    elif have < world:
        pytest.skip(f"needs {world} GPUs")
    m, k, n = 1000, 700, 1500
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    store_file = str(tmp_path / "store")
    procs = [ctx.Process(target=_worker, args=(r, world, store_file, m, k, n, q, transport)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    n2 = n // 2 + 1
    C = np.full((m, n), np.nan)
    C2 = np.full((m, n2), np.nan)
    for rank, status, payload in results:
        assert status == "ok", payload
        r0, r1, Cr, C2r, code = payload
        assert code[0] == 0, code
        C[r0:r1] = Cr
        C2[r0:r1] = C2r
    A, B = _problem(m, k, n)
    want = oo.ozaki2_matmul(A, B)
    np.testing.assert_array_equal(C.view(np.int64), want.view(np.int64))
    # Column exponents are per column, so the product with B[:, :n2] is C[:, :n2].
    np.testing.assert_array_equal(C2.view(np.int64), want[:, :n2].view(np.int64))


def _allgather_worker(rank, world, store_file, m, k, nb, q):
    try:
        import torch

        os.environ.update(NCCL_NVLS_ENABLE="0", FPEMU_CHUNK_COLS="256")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        torch.distributed.init_process_group("nccl", init_method=f"file://{store_file}", rank=rank,
                                             world_size=world, device_id=dev, timeout=timedelta(seconds=60))
        from fp_emulation import _lib
        from fp_emulation.distributed import ozaki2_int8_matmul_allgather, shard_rows

        A, B = _problem(m, k, world * nb)
        r0, r1 = shard_rows(m, world, rank)
        A_local = torch.from_numpy(A[r0:r1]).to(dev)
        B_local = torch.from_numpy(np.ascontiguousarray(B[:, rank * nb:(rank + 1) * nb])).to(dev)
        for _ in range(2):  # buffers, events and store keys reused by the second call
            C = ozaki2_int8_matmul_allgather(A_local, B_local)
        torch.cuda.synchronize(dev)
        code = _lib.device_error(clear=True)
        q.put((rank, "ok", (r0, r1, C.cpu().numpy(), code)))
        torch.distributed.barrier(device_ids=[rank])
        torch.distributed.destroy_process_group()
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


@pytest.mark.parametrize("world", [2, "all"])
def test_allgather_product_column_sharded_b_bit_exact(world, tmp_path):
    """A row-sharded, B column-sharded (rank q holds columns [q*nb, (q+1)*nb));
    blocks of 250 columns cut into strips of 256 // world columns, so the last
    chunk is narrower.  The gathered rows of C equal the oracle's full product."""
    import torch
    import torch.multiprocessing as mp

    have = torch.cuda.device_count()
    if world == "all":
        if have < 3:
            pytest.skip("needs 3 or more GPUs")
        world = have
    elif have < world:
        pytest.skip(f"needs {world} GPUs")
    m, k, nb = 900, 700, 250
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    store_file = str(tmp_path / "store")
    procs = [ctx.Process(target=_allgather_worker, args=(r, world, store_file, m, k, nb, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    C = np.full((m, world * nb), np.nan)
    for rank, status, payload in results:
        assert status == "ok", payload
        r0, r1, Cr, code = payload
        assert code[0] == 0, code
        C[r0:r1] = Cr
    A, B = _problem(m, k, world * nb)
    np.testing.assert_array_equal(C.view(np.int64), oo.ozaki2_matmul(A, B).view(np.int64))
