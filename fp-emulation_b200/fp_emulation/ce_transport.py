"""SM-free broadcast of B's residue chunks over NVLink, moved by the GPUs' copy
engines through CUDA IPC.

Why: NCCL's broadcast runs as kernels (about 24 GB/s per channel, one CTA per
channel), so at the 8-GPU point it needs ~27 SMs for the whole 10 ms it takes
to move B's 6.7 GB of residues -- SMs the persistent GEMM is using.  Copy
engines need no SMs, so the transfer hides under the tensor work.

Every rank owns one device buffer (cudaMalloc) holding B's residue chunks
(chunk c = int8 [n_mod][W][ld] followed by its W column exponents) and shares it
through CUDA IPC together with interprocess events.  Copies are pulls: the
receiving rank's stream copies from the peer's buffer into its own after waiting
on the peer's event.  A stream may only wait on an event after the peer has
enqueued the matching record, so ranks publish "phase enqueued" keys through the
process group's store and wait for the keys they depend on before enqueuing
waits.  All data movement and all GPU-side ordering is stream/event based; the
host only orders the enqueues.

The topology is a pipelined chain root -> next -> ... -> last, each chunk in
pieces: every GPU receives each byte once from one predecessor and sends it
once to one successor, which keeps every copy engine on one NVLink flow.  (A
scatter from the root followed by an all-gather, tried as well, ran at about
half the chain's bandwidth: a GPU pulling from six peers at once.)  The chain
is World-1 hops deep, so its fill latency grows with the rank count.
"""
from __future__ import annotations

import atexit
import mmap
import os
import time

import numpy as np
import torch
import torch.distributed as dist
from cuda.bindings import runtime as rt


def _check(res, what):
    err = res[0] if isinstance(res, tuple) else res
    if err != rt.cudaError_t.cudaSuccess:
        raise RuntimeError(f"{what} failed: {err}")
    return res[1] if isinstance(res, tuple) and len(res) == 2 else res


_SHM_DIR = "/dev/shm"  # node-local shared memory (tmpfs)


def _align256(x):
    return (x + 255) // 256 * 256


class _Ext:
    """A device allocation exposed to torch through __cuda_array_interface__."""

    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|i1", "data": (ptr, False),
                                         "version": 3}


class _IpcChunks:
    """The shared part: a chunked device buffer, named per-chunk interprocess
    events, handle exchange over the group, peers' buffers and events opened on
    demand, and the store keys that order the ranks' enqueues.

    Construction is collective over the group, so every rank builds its
    transports in the same order; the construction serial within the group (with
    the group's global ranks) names the store keys identically on every rank."""

    _serials: dict = {}
    EVENTS: tuple = ()

    def __init__(self, group, root, device, chunk_bytes, n_chunks, extra_bytes=0):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.root = root
        self.device = device
        self.n_chunks = n_chunks
        self.chunk_bytes = chunk_bytes
        self.store = dist.distributed_c10d._get_default_store()
        self.calls = 0
        members = tuple(dist.get_process_group_ranks(group)) if group is not None else ("world",)
        serial = _IpcChunks._serials.get(members, 0)
        _IpcChunks._serials[members] = serial + 1
        self.key_prefix = f"fpemu_ce/{'-'.join(map(str, members))}/{serial}"
        R = self._rt
        flags = R.cudaEventDisableTiming | R.cudaEventInterprocess
        with self._device_ctx():
            self.nbytes = chunk_bytes * n_chunks + extra_bytes
            self.ptr = _check(R.cudaMalloc(self.nbytes), "cudaMalloc")
            self.buf = self._wrap_buffer(int(self.ptr), self.nbytes)
            self.ev = {name: [_check(R.cudaEventCreateWithFlags(flags), "cudaEventCreate")
                              for _ in range(self._events_per_chunk(name) * n_chunks)]
                       for name in self.EVENTS}
            self.gemm_done = [self._local_event() for _ in range(n_chunks)]
            mem_h = bytes(_check(R.cudaIpcGetMemHandle(self.ptr), "cudaIpcGetMemHandle").reserved)
            ev_h = {name: [bytes(_check(R.cudaIpcGetEventHandle(e), "cudaIpcGetEventHandle").reserved)
                           for e in evs] for name, evs in self.ev.items()}
        self._table = [None] * self.world
        dist.all_gather_object(self._table, (mem_h, ev_h), group=group)
        self._peer_ptr = {}
        self._peer_ev = {}
        atexit.register(self.close)

    def _events_per_chunk(self, name):
        return 1

    # -- the CUDA runtime and torch objects this class touches.  Kept behind
    # these hooks so that the enqueue protocol can be exercised on the CPU with
    # a fake runtime (tests/test_ce_protocol.py); the defaults are the real ones.
    _rt = rt

    def _device_ctx(self):
        return torch.cuda.device(self.device)

    def _wrap_buffer(self, ptr, nbytes):
        return torch.as_tensor(_Ext(ptr, nbytes), device=self.device)

    def _local_event(self):
        return torch.cuda.Event()

    def _new_stream(self):
        return torch.cuda.Stream(self.device)

    def _current_stream(self):
        return torch.cuda.current_stream(self.device)

    def peer_ptr(self, r):
        if r not in self._peer_ptr:
            R = self._rt
            h = R.cudaIpcMemHandle_t()
            h.reserved = self._table[r][0]
            with self._device_ctx():
                self._peer_ptr[r] = int(_check(R.cudaIpcOpenMemHandle(h, R.cudaIpcMemLazyEnablePeerAccess),
                                               "cudaIpcOpenMemHandle"))
        return self._peer_ptr[r]

    def peer_events(self, r, name):
        if (r, name) not in self._peer_ev:
            R = self._rt
            evs = []
            with self._device_ctx():
                for hb in self._table[r][1][name]:
                    eh = R.cudaIpcEventHandle_t()
                    eh.reserved = hb
                    evs.append(_check(R.cudaIpcOpenEventHandle(eh), "cudaIpcOpenEventHandle"))
            self._peer_ev[(r, name)] = evs
        return self._peer_ev[(r, name)]

    def chunk_view(self, c):
        return self.buf[c * self.chunk_bytes:(c + 1) * self.chunk_bytes]

    def _key(self, rank, call, phase):
        return f"{self.key_prefix}/{call}/{phase}/{rank}"

    def _wait_keys(self, ranks, call, phase):
        keys = [self._key(r, call, phase) for r in ranks]
        if keys:
            self.store.wait(keys)

    def _publish(self, phase):
        self.store.set(self._key(self.rank, self.calls, phase), "1")

    def _forget(self, call, phases):
        """Delete this rank's keys of an old call once no rank can still wait on them."""
        if call >= 0:
            for ph in phases:
                self.store.delete_key(self._key(self.rank, call, ph))

    def _wait(self, stream, event, what="wait"):
        _check(self._rt.cudaStreamWaitEvent(stream.cuda_stream, event, 0), what)

    def _record(self, stream, event):
        _check(self._rt.cudaEventRecord(event, stream.cuda_stream), "record")

    def _copy(self, stream, dst, src, nbytes):
        _check(self._rt.cudaMemcpyAsync(dst, src, nbytes, self._rt.cudaMemcpyKind.cudaMemcpyDeviceToDevice,
                                        stream.cuda_stream), "memcpy")

    def _copy2d(self, stream, dst, dpitch, src, spitch, width, height):
        _check(self._rt.cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, height,
                                          self._rt.cudaMemcpyKind.cudaMemcpyDeviceToDevice, stream.cuda_stream),
               "memcpy2d")

    def after_gemm(self, c, stream):
        """This rank's GEMM on chunk c is enqueued on `stream`: the chunk may be
        overwritten by the next call once it has run."""
        self.gemm_done[c].record(stream)

    def _drain(self):
        torch.cuda.synchronize(self.device)

    def _phases(self):
        return ("A",)

    def release(self, barrier):
        """Free the buffer and the events.  Collective: every rank of the group
        releases the same transport in the same call; `barrier()` meets them.
        This device drains first; after the first meeting no rank has work on
        any buffer of this transport, after the second no peer maps this one."""
        R = self._rt
        self._drain()
        barrier()
        for ptr in self._peer_ptr.values():
            _check(R.cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle")
        for evs in self._peer_ev.values():
            for e in evs:
                _check(R.cudaEventDestroy(e), "cudaEventDestroy")
        self._peer_ptr, self._peer_ev = {}, {}
        for i in (self.calls - 2, self.calls - 1):  # nobody waits on these any more
            self._forget(i, self._phases())
        barrier()
        for evs in self.ev.values():
            for e in evs:
                _check(R.cudaEventDestroy(e), "cudaEventDestroy")
        self.ev = {}
        _check(R.cudaFree(self.ptr), "cudaFree")
        self.ptr, self.buf = None, None
        atexit.unregister(self.close)

    def close(self):
        for ptr in self._peer_ptr.values():
            try:
                self._rt.cudaIpcCloseMemHandle(ptr)
            except Exception:
                pass
        self._peer_ptr = {}


class CeChain(_IpcChunks):
    """Pipelined chain root -> next -> ... -> last; each chunk moves in `pieces`
    pieces, rank r copying piece (c, q) from its predecessor as soon as the
    predecessor's ``done[c][q]`` fires.  Phase "A" = all of this call's records
    enqueued; a rank waits for its predecessor's "A" of this call before
    enqueuing waits on it, and for its successor's "A" of the previous call
    before overwriting what the successor read."""

    EVENTS = ("done",)

    def __init__(self, group, root, device, chunk_bytes, n_chunks, pieces=None):
        self.pieces = int(os.environ.get("FPEMU_CE_PIECES", "8")) if pieces is None else pieces
        super().__init__(group, root, device, chunk_bytes, n_chunks)
        order = [(root + i) % self.world for i in range(self.world)]
        pos = order.index(self.rank)
        self.pred = order[pos - 1] if pos > 0 else None
        self.succ = order[pos + 1] if pos + 1 < self.world else None
        self.split_stream = self._current_stream()
        self.copy_stream = self._new_stream()

    def _events_per_chunk(self, name):
        return self.pieces

    def _done(self, r, c, q):
        evs = self.ev["done"] if r == self.rank else self.peer_events(r, "done")
        return evs[c * self.pieces + q]

    def _piece(self, q):
        step = _align256(-(-self.chunk_bytes // self.pieces))
        lo = min(q * step, self.chunk_bytes)
        return lo, min(self.chunk_bytes, lo + step)

    # Store keys of old calls: key (r, i) is waited on by r's successor in call i
    # and by r's predecessor in call i+1.  When r has passed its own key waits of
    # call i+2 -- its predecessor's key of i+2 and its successor's of i+1, each
    # published after that rank's waits of the earlier call -- both neighbours
    # are done with (r, i), so r deletes it then.

    def root_begin(self, main_stream):
        if self.calls > 0 and self.succ is not None:
            self._wait_keys([self.succ], self.calls - 1, "A")
        self._forget(self.calls - 2, ("A",))
        self.split_stream = main_stream

    def root_before_write(self, c):
        if self.calls > 0 and self.succ is not None:
            for q in range(self.pieces):
                self._wait(self.split_stream, self._done(self.succ, c, q))

    def root_after_write(self, c):
        for q in range(self.pieces):
            self._record(self.split_stream, self._done(self.rank, c, q))

    def root_end(self):
        self._publish("A")
        self.calls += 1

    def pull(self):
        i = self.calls
        if i > 0 and self.succ is not None:
            self._wait_keys([self.succ], i - 1, "A")
        self._wait_keys([self.pred], i, "A")
        self._forget(i - 2, ("A",))
        cs = self.copy_stream
        pred_ptr = self.peer_ptr(self.pred)
        for c in range(self.n_chunks):
            cs.wait_event(self.gemm_done[c])
            base = c * self.chunk_bytes
            for q in range(self.pieces):
                lo, hi = self._piece(q)
                self._wait(cs, self._done(self.pred, c, q), "wait pred")
                if i > 0 and self.succ is not None:
                    self._wait(cs, self._done(self.succ, c, q), "wait succ")
                if hi > lo:
                    self._copy(cs, int(self.ptr) + base + lo, pred_ptr + base + lo, hi - lo)
                self._record(cs, self._done(self.rank, c, q))
        self._publish("A")
        self.calls += 1

    def wait_chunk(self, c, stream):
        self._wait(stream, self._done(self.rank, c, self.pieces - 1), "wait chunk")


class _Positions:
    """How far each rank of the group has enqueued its transport work: one
    monotonic int64 per rank in a shared-memory block that every rank of the
    node maps (the products run one process per GPU on one node).  A rank
    publishes the position of each item after enqueuing it; a rank about to
    enqueue a stream wait on a peer's event first waits until the peer's
    position shows that the matching record is enqueued.  Reading a shared word
    costs about a microsecond where a store round trip costs tens, so the ring
    can order its enqueues per (chunk, step).  Host waits are bounded
    (FPEMU_HOST_WAIT_S, default 120 s) and raise instead of hanging."""

    def __init__(self, group, rank, world, tag):
        self.rank = rank
        self.timeout = float(os.environ.get("FPEMU_HOST_WAIT_S", "120"))
        name = f"fpemu_pos_{os.getpid()}_{tag}"
        self._path = os.path.join(_SHM_DIR, name)
        own = self._map(self._path, create=True)
        np.ndarray((1,), dtype=np.int64, buffer=own)[0] = -1
        names = [None] * world
        dist.all_gather_object(names, name, group=group)
        self._maps = [own if r == rank else self._map(os.path.join(_SHM_DIR, n)) for r, n in enumerate(names)]
        self._views = [np.ndarray((1,), dtype=np.int64, buffer=m) for m in self._maps]
        atexit.register(self.close)

    @staticmethod
    def _map(path, create=False):
        # Plain files in the node's shared-memory file system, mapped directly:
        # multiprocessing's SharedMemory would register peers' blocks with each
        # process's resource tracker as if that process owned them.  Only the
        # creating rank unlinks its block.
        flags = os.O_RDWR | (os.O_CREAT | os.O_EXCL if create else 0)
        try:
            fd = os.open(path, flags, 0o600)
        except FileExistsError:
            # Names carry the creator's pid and a per-process serial, so an
            # existing file was left by a dead process that had this pid.
            os.unlink(path)
            fd = os.open(path, flags, 0o600)
        try:
            if create:
                os.ftruncate(fd, 8)
            return mmap.mmap(fd, 8)
        finally:
            os.close(fd)

    def publish(self, pos):
        self._views[self.rank][0] = pos

    def wait(self, r, pos, what=""):
        v = self._views[r]
        if v[0] >= pos:
            return
        t0 = time.monotonic()
        while v[0] < pos:
            if time.monotonic() - t0 > self.timeout:
                raise RuntimeError(f"rank {self.rank}: rank {r} did not enqueue {what} (position {pos}, at {v[0]}) "
                                   f"within {self.timeout:.0f} s")
            time.sleep(2e-5)

    def close(self):
        views, self._views = self._views, []
        del views
        for m in self._maps:
            try:
                m.close()
            except Exception:
                pass
        self._maps = []
        try:
            os.unlink(self._path)
        except OSError:
            pass


class CeRing(_IpcChunks):
    """Every rank splits one strip of each chunk; the residue strips then go
    round a ring by the copy engines, chunk after chunk.

    Ranks form the ring order = root, root+1, ...; pred/succ are the neighbours
    in it.  Per call, for each chunk c in order:
      root, copy stream:   (staged) FP64 strip q of B -> rank q's staging slot c
                           (2-D copy into the peer's buffer), then record stage[c];
      rank r, split stream: (staged: after the root's stage[c]) split its own
                           strip into its residue buffer, record have[c][r];
      rank r, ring stream: for step t = 1 .. W-1, the strip s that is t positions
                           behind r is in pred's buffer once pred's have[c][s]
                           fires (pred's split for t = 1, its step t-1
                           otherwise): copy it, in `pieces` groups of modulus
                           planes, each recorded as have[c][s][piece];
      GEMM on chunk c:     after have[c][q] for every q.
    All steps of a chunk go before the next chunk on the one ring stream, so
    every hop of chunk c has the link to itself: chunk 0 arrives after W-1 hops
    (in pieces) and the others follow one per chunk transfer time, instead of
    all chunks advancing together and arriving together.
    Reuse across calls: the root overwrites slot c after every rank's split of
    the previous call read it; r overwrites its strip s of chunk c after its own
    GEMM of the previous call and, unless s is succ's own strip, after succ
    pulled it.
    Host order: item (call, c, k) -- k = 0 stage, 1 split, 1 + t ring step t --
    has position ((call * chunks) + c) * (W + 1) + k; each rank publishes its
    position after enqueuing an item (_Positions) and, before enqueuing a wait
    on a peer's record, waits until the peer has published the item holding that
    record.  Every wait points to an item of an earlier chunk, an earlier step of
    the same chunk on the predecessor, or the previous call, so the ranks never
    wait in a circle, and the peer cannot enqueue its next record of an event
    before this rank has enqueued its wait on the current one."""

    EVENTS = ("stage", "have")

    def __init__(self, group, root, device, layout, staged=True, pieces=None):
        """staged=False: no root staging -- every rank splits its strips from its
        own copy of its part of B (a column-sharded B), and only the ring moves
        data between GPUs.  `pieces` (FPEMU_RING_PIECES, default 1): each ring
        step moves a strip as that many groups of modulus planes, each with its
        own event, so the next hop can start on the first group.  One piece is
        the default: every piece costs an interprocess-event handshake (tens of
        microseconds on the copy stream), and the ring's steps run in lockstep,
        so a whole-strip dependency between steps costs little (4 GPUs,
        column-sharded B, n = 16384: 21.2 ms with 1 piece, 21.8 ms with 4)."""
        self.layout = layout
        self.staged = staged
        P = int(os.environ.get("FPEMU_RING_PIECES", "1")) if pieces is None else pieces
        self.pieces = max(1, min(layout.n_mod, P))
        nc = len(layout.plan)
        super().__init__(group, root, device, layout.chunk_bytes, nc, extra_bytes=nc * layout.slot_bytes)
        W = self.world
        self.order = [(root + i) % W for i in range(W)]
        self.pos = self.order.index(self.rank)
        self.pred = self.order[(self.pos - 1) % W]
        self.succ = self.order[(self.pos + 1) % W]
        self.split_stream = self._new_stream()
        self.copy_stream = self._new_stream()
        self.ring_stream = self._new_stream()
        self.board = self._positions(group)

    def _positions(self, group):
        return _Positions(group, self.rank, self.world, self.key_prefix.replace("/", "_"))

    def _events_per_chunk(self, name):
        return self.world * self.pieces if name == "have" else 1

    def _phases(self):
        return ()

    def _have(self, owner, c, q, p=None):
        """Event `owner` records once piece p of strip q of chunk c is in its buffer;
        p defaults to the last piece, recorded after all the others on the same stream."""
        p = self.pieces - 1 if p is None else p
        evs = self.ev["have"] if owner == self.rank else self.peer_events(owner, "have")
        return evs[(c * self.world + q) * self.pieces + p]

    def plane_pieces(self):
        """[(first plane, end plane)] of each piece: n_mod planes in near-equal groups."""
        n, P = self.layout.n_mod, self.pieces
        return [(p * n // P, (p + 1) * n // P) for p in range(P)]

    def _stage(self, c):
        evs = self.ev["stage"] if self.rank == self.root else self.peer_events(self.root, "stage")
        return evs[c]

    def strip_at(self, t):
        """The strip (by owning rank) that reaches this rank at ring step t."""
        return self.order[(self.pos - t) % self.world]

    def _base(self, r):
        return int(self.ptr) if r == self.rank else self.peer_ptr(r)

    def _at(self, call, c, k):
        return (call * len(self.layout.plan) + c) * (self.world + 1) + k

    # -- per call ---------------------------------------------------------------
    def enqueue(self, split_fn, main_stream, B_ptr=None, ldb=None):
        """Enqueue this call's transport: per chunk, the root's staging (staged:
        B_ptr/ldb, the root's row-major B), every rank's split of its strip
        (split_fn(c, stream) enqueues it on `stream`), and the ring steps.  The
        split stream (unstaged) and the root's copy stream (staged) first wait for
        `main_stream`, where the caller produced B."""
        i = self.calls
        L = self.layout
        W = self.world
        board, at = self.board, self._at
        ss, rs, cs = self.split_stream, self.ring_stream, self.copy_stream
        if self.staged and self.rank == self.root:
            cs.wait_stream(main_stream)
        if not self.staged:
            ss.wait_stream(main_stream)
        pieces = self.plane_pieces()
        for c, (c0, c1) in enumerate(L.plan):
            w = c1 - c0
            base = c * L.chunk_bytes
            # Root: this chunk's FP64 strips into every rank's staging slot c.
            if self.staged and self.rank == self.root:
                if i > 0:
                    for q in range(W):
                        board.wait(q, at(i - 1, c, 1), "its previous split")
                        self._wait(cs, self._have(q, c, q), "stage war")
                for q, (s0, s1) in enumerate(L.strips[c]):
                    if s1 > s0:
                        self._copy2d(cs, self._base(q) + L.stage_off + c * L.slot_bytes, L.pitch * 8,
                                     B_ptr + (c0 + s0) * 8, ldb * 8, (s1 - s0) * 8, L.k)
                self._record(cs, self._stage(c))
                board.publish(at(i, c, 0))
            # Every rank: split its own strip of chunk c.
            ss.wait_event(self.gemm_done[c])
            if self.staged:
                board.wait(self.root, at(i, c, 0), "the staging")
                self._wait(ss, self._stage(c), "stage")
            if i > 0 and W > 1:  # succ pulled this strip at its step 1 of the previous call
                board.wait(self.succ, at(i - 1, c, 2), "its previous step 1")
                self._wait(ss, self._have(self.succ, c, self.rank), "split war")
            split_fn(c, ss)
            for p in range(self.pieces):  # the split wrote every piece of this rank's strip
                self._record(ss, self._have(self.rank, c, self.rank, p))
            board.publish(at(i, c, 1))
            # Every rank: the W-1 other strips of chunk c round the ring.
            if W > 1:
                rs.wait_event(self.gemm_done[c])
            for t in range(1, W):
                s = self.strip_at(t)
                board.wait(self.pred, at(i, c, 1 if t == 1 else t), f"step {t - 1} of chunk {c}")
                war = i > 0 and t < W - 1  # succ pulls this strip from us at its step t+1
                if war:
                    board.wait(self.succ, at(i - 1, c, t + 2), f"its previous step {t + 1}")
                s0, s1 = L.strips[c][s]
                for p, (l0, l1) in enumerate(pieces):
                    self._wait(rs, self._have(self.pred, c, s, p), "ring")
                    if war:
                        self._wait(rs, self._have(self.succ, c, s, p), "ring war")
                    if s1 > s0:
                        # residues: rows s0..s1 of planes l0..l1 (plane stride w*ld)
                        off = base + l0 * w * L.ld + s0 * L.ld
                        self._copy2d(rs, int(self.ptr) + off, w * L.ld, self.peer_ptr(self.pred) + off, w * L.ld,
                                     (s1 - s0) * L.ld, l1 - l0)
                        if p == len(pieces) - 1:
                            off = base + L.res_bytes + 4 * s0  # column exponents
                            self._copy(rs, int(self.ptr) + off, self.peer_ptr(self.pred) + off, 4 * (s1 - s0))
                    self._record(rs, self._have(self.rank, c, s, p))
                board.publish(at(i, c, 1 + t))
        self.calls += 1

    def wait_chunk(self, c, stream):
        """`stream` waits until every strip of chunk c is in this rank's buffer."""
        for q in range(self.world):
            self._wait(stream, self._have(self.rank, c, q), "gemm")

    def release(self, barrier):
        super().release(barrier)
        if self.board is not None:
            self.board.close()
            self.board = None

    def close(self):
        super().close()
        board = getattr(self, "board", None)
        if board is not None:
            board.close()
            self.board = None


TRANSPORTS = {"ce": CeChain, "ce-ring": CeRing}
