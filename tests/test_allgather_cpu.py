"""The column-sharded multi-GPU product (distributed.rowsharded_product_allgather)
end to end on CPU ranks: gloo process groups, a fake CUDA runtime that really
moves the bytes -- each rank's transport buffer is a shared-memory block that
the peers map in place of CUDA IPC, every copy the ring enqueues is done at once
-- and a CPU backend whose split and segmented GEMM + CRT come from the oracle.

Executing every enqueued copy immediately is faithful to the transport's
ordering: a rank enqueues a copy from a peer only after the peer published the
phase whose records mark that data as written, and overwrites a strip only
after the reader published the phase that pulled it.  So the test checks the
data path -- which rank splits which strip, where the ring puts it, which
columns of C each chunk's GEMM writes -- bit for bit against the oracle's full
product, for 2 and 3 ranks, two calls in a row, and a ragged last chunk.
"""
from __future__ import annotations

import contextlib
import os
import socket
import traceback
from datetime import timedelta
from multiprocessing import shared_memory

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from cuda.bindings import runtime as _real_rt
from oracle import ozaki_oracle as oo

OK = _real_rt.cudaError_t.cudaSuccess
SPAN = 0x10000000  # fake device addresses: rank r's buffer at (r + 1) * SPAN


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _Handle:
    def __init__(self, reserved=b""):
        self.reserved = reserved


class MemRt:
    """The runtime calls of the transport, on shared-memory buffers."""

    cudaEventDisableTiming = 2
    cudaEventInterprocess = 4
    cudaIpcMemLazyEnablePeerAccess = 1
    cudaIpcMemHandle_t = _Handle
    cudaIpcEventHandle_t = _Handle

    class cudaMemcpyKind:
        cudaMemcpyDeviceToDevice = 3

    def __init__(self, rank, tag):
        self.rank, self.tag = rank, tag
        self.shm = {}
        self.n_events = 0

    def cudaMalloc(self, nbytes):
        shm = shared_memory.SharedMemory(create=True, size=nbytes, name=f"{self.tag}_{self.rank}")
        base = SPAN * (self.rank + 1)
        self.shm[base] = shm
        return OK, base

    def cudaIpcGetMemHandle(self, ptr):
        return OK, _Handle(f"{self.tag}_{self.rank}|{self.rank}".encode())

    def cudaIpcOpenMemHandle(self, h, flags):
        name, r = h.reserved.decode().split("|")
        base = SPAN * (int(r) + 1)
        self.shm[base] = shared_memory.SharedMemory(name=name)
        return OK, base

    def _view(self, addr, n):
        base = addr - addr % SPAN
        return np.frombuffer(self.shm[base].buf, dtype=np.uint8, count=n, offset=addr - base)

    def cudaMemcpyAsync(self, dst, src, nbytes, kind, stream):
        self._view(dst, nbytes)[:] = self._view(src, nbytes)
        return (OK,)

    def cudaMemcpy2DAsync(self, dst, dpitch, src, spitch, width, height, kind, stream):
        for r in range(height):
            self._view(dst + r * dpitch, width)[:] = self._view(src + r * spitch, width)
        return (OK,)

    def cudaEventCreateWithFlags(self, flags):
        self.n_events += 1
        return OK, (self.rank, self.n_events - 1)

    def cudaIpcGetEventHandle(self, ev):
        return OK, _Handle(f"{ev[0]}:{ev[1]}".encode())

    def cudaIpcOpenEventHandle(self, h):
        owner, idx = h.reserved.decode().split(":")
        return OK, (int(owner), int(idx))

    def cudaEventRecord(self, ev, stream):
        return (OK,)

    def cudaStreamWaitEvent(self, stream, ev, flags):
        return (OK,)

    def cudaIpcCloseMemHandle(self, ptr):
        return (OK,)

    def cudaEventDestroy(self, ev):
        return (OK,)

    def cudaFree(self, ptr):
        return (OK,)


class _Stream:
    cuda_stream = 0

    def wait_event(self, ev):
        pass

    def wait_stream(self, other):
        pass


class _LocalEvent:
    def record(self, stream=None):
        pass


class OracleOps:
    """CPU stand-in for the GPU backend: the oracle's split and GEMM + CRT."""

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

    def gemm_crt_segmented(self, a_res, re, b_res, ce_chunk, bits, C, col_off, seg, seg_stride, k):
        n_mod = a_res.shape[0]
        moduli = oo.PRIMES[:n_mod]
        res = oo.matmul_residues(a_res[:, :, :k].numpy(), b_res[:, :, :k].numpy().transpose(0, 2, 1), moduli)
        vals = oo.reconstruct(res, moduli, bits, re.numpy(), ce_chunk.numpy())
        j = np.arange(vals.shape[1])
        C[:, col_off + (j // seg) * seg_stride + j % seg] = torch.from_numpy(vals)


def _problem(m, k, n):
    rng = np.random.default_rng(31)
    A = (rng.random((m, k)) - 0.5) * np.exp(rng.standard_normal((m, k)))
    B = (rng.random((k, n)) - 0.5) * np.exp(rng.standard_normal((k, n)))
    return A, B


def _worker(rank, world, port, m, k, nb, strip, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import torch.distributed as dist

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        import fp_emulation.ce_transport as ct
        from fp_emulation import distributed as fd

        rt = MemRt(rank, f"fpemu_ag_{port}")
        Ring = ct.CeRing

        class MemRing(Ring):
            _rt = rt

            def _device_ctx(self):
                return contextlib.nullcontext()

            def _wrap_buffer(self, ptr, nbytes):
                return torch.frombuffer(rt.shm[ptr].buf, dtype=torch.uint8, count=nbytes)

            def _local_event(self):
                return _LocalEvent()

            def _new_stream(self):
                return _Stream()

            def _current_stream(self):
                return _Stream()

        ct.CeRing = MemRing
        torch.cuda.current_stream = lambda device=None: _Stream()
        torch.cuda.stream = lambda s: contextlib.nullcontext()
        torch.Tensor.record_stream = lambda self, s: None

        A, B = _problem(m, k, world * nb)
        r0, r1 = fd.shard_rows(m, world, rank)
        A_local = torch.from_numpy(A[r0:r1])
        B_local = torch.from_numpy(np.ascontiguousarray(B[:, rank * nb:(rank + 1) * nb]))
        n_mod = oo.n_moduli(k, 53)
        outs = [fd.rowsharded_product_allgather(A_local, B_local, k, 53, n_mod, OracleOps(), strip_cols=strip)
                .numpy().copy() for _ in range(2)]
        q.put((rank, "ok", (r0, r1, outs)))
        dist.barrier()
        for shm in rt.shm.values():
            shm.close()
        own = rt.shm.get(SPAN * (rank + 1))
        if own is not None:
            own.unlink()
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


@pytest.mark.parametrize("world,nb,strip", [(2, 50, 16), (3, 33, 16)])
def test_allgather_product_on_cpu_ranks_matches_the_oracle(world, nb, strip):
    m, k = 80, 70
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, m, k, nb, strip, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    A, B = _problem(m, k, world * nb)
    want = oo.ozaki2_matmul(A, B)
    for call in range(2):
        C = np.full(want.shape, np.nan)
        for rank, status, payload in results:
            assert status == "ok", payload
            r0, r1, outs = payload
            C[r0:r1] = outs[call]
        np.testing.assert_array_equal(C.view(np.int64), want.view(np.int64))
