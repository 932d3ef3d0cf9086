"""SM-free broadcast of B's residue chunks over NVLink: a pipelined chain
root -> next -> ... -> last, moved by the GPUs' copy engines.

Why: NCCL's broadcast runs as kernels (about 24 GB/s per channel, one CTA per
channel), so at the 8-GPU point it needs ~27 SMs for the whole 10 ms it takes
to move B's 6.7 GB of residues -- SMs the persistent GEMM is using.  Copy
engines need no SMs, so the transfer hides under the tensor work.

How: every rank owns one device buffer (cudaMalloc) holding B's residue
chunks (chunk c = int8 [n_mod][W][ld] followed by its W column exponents), and
shares it with its chain neighbours through CUDA IPC.  A chunk moves in pieces;
rank r copies piece (c, q) from its predecessor's buffer into its own as soon
as the predecessor's interprocess event `done[c][q]` fires, then records its
own `done[c][q]` (which the successor waits on, and which also tells the
predecessor, in the next call, that the piece may be overwritten).  Each wait
must be enqueued after the matching record, so ranks publish "call i enqueued"
through the process group's store and wait for their predecessor's key (and,
before overwriting, their successor's key from the previous call).  The last
rank's copies and everyone's GEMMs follow purely from stream events.
"""
from __future__ import annotations

import atexit

import torch
import torch.distributed as dist
from cuda.bindings import runtime as rt


def _check(res, what):
    err = res[0] if isinstance(res, tuple) else res
    if err != rt.cudaError_t.cudaSuccess:
        raise RuntimeError(f"{what} failed: {err}")
    return res[1] if isinstance(res, tuple) and len(res) == 2 else res


class _Ext:
    """A device allocation exposed to torch through __cuda_array_interface__."""

    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|i1", "data": (ptr, False),
                                         "version": 3}


class CeChain:
    """One chain broadcast channel for a fixed chunk layout (reused across calls)."""

    def __init__(self, group, root, device, chunk_bytes, n_chunks, pieces=8):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.root = root
        self.device = device
        self.n_chunks = n_chunks
        self.pieces = pieces
        self.chunk_bytes = chunk_bytes
        self.store = dist.distributed_c10d._get_default_store()
        self.calls = 0
        order = [(root + i) % self.world for i in range(self.world)]
        pos = order.index(self.rank)
        self.pred = order[pos - 1] if pos > 0 else None
        self.succ = order[pos + 1] if pos + 1 < self.world else None
        with torch.cuda.device(device):
            self.nbytes = chunk_bytes * n_chunks
            self.ptr = _check(rt.cudaMalloc(self.nbytes), "cudaMalloc")
            self.buf = torch.as_tensor(_Ext(int(self.ptr), self.nbytes), device=device)
            flags = rt.cudaEventDisableTiming | rt.cudaEventInterprocess
            self.done = [[_check(rt.cudaEventCreateWithFlags(flags), "cudaEventCreate") for _ in range(pieces)]
                         for _ in range(n_chunks)]
            self.gemm_done = [torch.cuda.Event() for _ in range(n_chunks)]
            self.copy_stream = torch.cuda.Stream(device)
            mem_h = bytes(_check(rt.cudaIpcGetMemHandle(self.ptr), "cudaIpcGetMemHandle").reserved)
            ev_h = [[bytes(_check(rt.cudaIpcGetEventHandle(e), "cudaIpcGetEventHandle").reserved) for e in row]
                    for row in self.done]
        table = [None] * self.world
        dist.all_gather_object(table, (mem_h, ev_h), group=group)
        self.pred_ptr = None
        self.pred_done = self.succ_done = None
        with torch.cuda.device(device):
            if self.pred is not None:
                h = rt.cudaIpcMemHandle_t()
                h.reserved = table[self.pred][0]
                self.pred_ptr = _check(rt.cudaIpcOpenMemHandle(h, rt.cudaIpcMemLazyEnablePeerAccess),
                                       "cudaIpcOpenMemHandle")
                self.pred_done = self._open_events(table[self.pred][1])
            if self.succ is not None:
                self.succ_done = self._open_events(table[self.succ][1])
        atexit.register(self.close)

    def _open_events(self, handles):
        out = []
        for row in handles:
            evs = []
            for hb in row:
                eh = rt.cudaIpcEventHandle_t()
                eh.reserved = hb
                evs.append(_check(rt.cudaIpcOpenEventHandle(eh), "cudaIpcOpenEventHandle"))
            out.append(evs)
        return out

    def chunk_view(self, c):
        return self.buf[c * self.chunk_bytes:(c + 1) * self.chunk_bytes]

    def _piece(self, q):
        step = ((self.chunk_bytes + self.pieces - 1) // self.pieces + 255) // 256 * 256
        lo = min(q * step, self.chunk_bytes)
        return lo, min(self.chunk_bytes, lo + step)

    def _key(self, rank, call):
        return f"fpemu_ce/{id(self.group) if self.group is not None else 0}/{call}/{rank}"

    # -- per call ---------------------------------------------------------
    def begin(self):
        """Host-side ordering before this call touches the buffer: the successor
        must have enqueued its reads of the previous call."""
        i = self.calls
        if i > 0 and self.succ is not None:
            self.store.wait([self._key(self.succ, i - 1)])

    def root_before_write(self, c, stream):
        """Root, before writing chunk c on `stream`: the successor has read the previous
        call's chunk c, and this rank's previous GEMM on it is done (same stream)."""
        if self.calls > 0 and self.succ is not None:
            for q in range(self.pieces):
                _check(rt.cudaStreamWaitEvent(stream.cuda_stream, self.succ_done[c][q], 0), "wait")

    def root_after_write(self, c, stream):
        for q in range(self.pieces):
            _check(rt.cudaEventRecord(self.done[c][q], stream.cuda_stream), "record")

    def relay(self):
        """Non-root: pull every piece from the predecessor on the copy stream."""
        i = self.calls
        self.store.wait([self._key(self.pred, i)])
        cs = self.copy_stream
        for c in range(self.n_chunks):
            cs.wait_event(self.gemm_done[c])  # this rank's previous GEMM has read chunk c
            base = c * self.chunk_bytes
            for q in range(self.pieces):
                lo, hi = self._piece(q)
                if hi <= lo:
                    _check(rt.cudaEventRecord(self.done[c][q], cs.cuda_stream), "record")
                    continue
                _check(rt.cudaStreamWaitEvent(cs.cuda_stream, self.pred_done[c][q], 0), "wait pred")
                if i > 0 and self.succ is not None:
                    _check(rt.cudaStreamWaitEvent(cs.cuda_stream, self.succ_done[c][q], 0), "wait succ")
                _check(rt.cudaMemcpyAsync(int(self.ptr) + base + lo, int(self.pred_ptr) + base + lo, hi - lo,
                                          rt.cudaMemcpyKind.cudaMemcpyDeviceToDevice, cs.cuda_stream), "memcpy")
                _check(rt.cudaEventRecord(self.done[c][q], cs.cuda_stream), "record")

    def wait_chunk(self, c, stream):
        """`stream` waits until chunk c is in this rank's buffer."""
        if self.rank != self.root:
            _check(rt.cudaStreamWaitEvent(stream.cuda_stream, self.done[c][self.pieces - 1], 0), "wait chunk")

    def after_gemm(self, c, stream):
        self.gemm_done[c].record(stream)

    def publish(self):
        self.store.set(self._key(self.rank, self.calls), "1")
        self.calls += 1

    def close(self):
        try:
            if self.pred_ptr is not None:
                rt.cudaIpcCloseMemHandle(self.pred_ptr)
                self.pred_ptr = None
        except Exception:
            pass
