"""The multi-GPU products of fp_emulation.distributed end to end on CPU ranks --
the column-sharded product (rowsharded_product_allgather) and the root-held
products over the copy-engine ring and chain: gloo process groups, a fake CUDA runtime that really
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
import ctypes
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
# Fake device addresses: rank r's buffer at BASE + r * SPAN, far from where a
# process maps its own memory (the ring also copies from the root's host B).
BASE = 0x100000000000
SPAN = 0x10000000


def _fake_base(r):
    return BASE + r * SPAN


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
        base = _fake_base(self.rank)
        self.shm[base] = shm
        return OK, base

    def cudaIpcGetMemHandle(self, ptr):
        return OK, _Handle(f"{self.tag}_{self.rank}|{self.rank}".encode())

    def cudaIpcOpenMemHandle(self, h, flags):
        name, r = h.reserved.decode().split("|")
        base = _fake_base(int(r))
        self.shm[base] = shared_memory.SharedMemory(name=name)
        return OK, base

    def _view(self, addr, n):
        for base, shm in self.shm.items():
            if base <= addr and addr + n <= base + shm.size:
                return np.frombuffer(shm.buf, dtype=np.uint8, count=n, offset=addr - base)
        # Any other address is host memory of this process (the root's B, staged by the ring).
        return np.ctypeslib.as_array((ctypes.c_uint8 * n).from_address(addr))

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

    def gemm_crt(self, a_res, re, b_res, ce_chunk, bits, C, c0, c1, k):
        self.gemm_crt_segmented(a_res, re, b_res, ce_chunk, bits, C, c0, c1 - c0, c1 - c0, k)

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


def _worker(rank, world, port, m, k, nb, strip, q, transport="allgather"):
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

        class MemChain(ct.CeChain):
            _rt = rt
            _device_ctx = MemRing._device_ctx
            _wrap_buffer = MemRing._wrap_buffer
            _local_event = MemRing._local_event
            _new_stream = MemRing._new_stream
            _current_stream = MemRing._current_stream

        ct.CeRing = MemRing
        ct.TRANSPORTS = {"ce": MemChain, "ce-ring": MemRing}
        torch.cuda.current_stream = lambda device=None: _Stream()
        torch.cuda.stream = lambda s: contextlib.nullcontext()
        torch.Tensor.record_stream = lambda self, s: None

        A, B = _problem(m, k, world * nb)
        r0, r1 = fd.shard_rows(m, world, rank)
        A_local = torch.from_numpy(A[r0:r1])
        B_local = torch.from_numpy(np.ascontiguousarray(B[:, rank * nb:(rank + 1) * nb]))
        n_mod = oo.n_moduli(k, 53)
        B_root = torch.from_numpy(B) if rank == 0 else None
        n = world * nb

        def product():
            if transport == "allgather":
                return fd.rowsharded_product_allgather(A_local, B_local, k, 53, n_mod, OracleOps(), strip_cols=strip)
            if transport == "ce-ring":
                return fd.rowsharded_product_ring(A_local, B_root, n, k, 53, n_mod, OracleOps(), chunk_cols=strip)
            return fd.rowsharded_product_ce(A_local, B_root, n, k, 53, n_mod, OracleOps(), chunk_cols=strip,
                                            transport="ce")

        outs = [product().numpy().copy() for _ in range(2)]
        q.put((rank, "ok", (r0, r1, outs)))
        dist.barrier()
        for shm in rt.shm.values():
            shm.close()
        own = rt.shm.get(_fake_base(rank))
        if own is not None:
            own.unlink()
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


@pytest.mark.parametrize("transport,world,nb,strip", [("allgather", 2, 50, 16), ("allgather", 3, 33, 16),
                                                     ("ce-ring", 2, 50, 256), ("ce-ring", 3, 100, 256),
                                                     ("ce", 3, 100, 256)])
def test_multi_gpu_products_on_cpu_ranks_match_the_oracle(transport, world, nb, strip):
    """allgather: column-sharded B (strips of `strip` columns).  ce-ring and ce: B on
    rank 0, chunks of `strip` columns (the ring stages FP64 strips from the root's
    B, splits them on every rank and circulates the residues; the chain has the
    root split every chunk and relays it in pieces)."""
    m, k = 80, 70
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, m, k, nb, strip, q, transport))
             for r in range(world)]
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
