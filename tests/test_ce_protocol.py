"""The copy-engine chain's enqueue protocol (fp_emulation/ce_transport.py) on
CPU ranks (gloo, one process per rank), with a fake CUDA runtime.

A stream may wait on a peer's interprocess event only after the peer has
enqueued the matching record -- and before it enqueues the next one, or the
wait binds to the wrong call.  The fake runtime counts every record of every
event in the process group's store at the moment it is enqueued, and logs, for
every stream wait, the count it saw.  The protocol is right when, in call i,
each wait on the predecessor's ``done`` saw exactly i+1 records (this call's),
each wait on the successor's ``done`` exactly i (the previous call's: the
successor has read it, and not yet begun the next), and each wait on the rank's
own ``done`` exactly i+1 -- for 2 to 4 ranks, roots other than rank 0, and
several calls in a row.  Old store keys must be deleted as calls go by.
"""
from __future__ import annotations

import contextlib
import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch.multiprocessing as mp

from cuda.bindings import runtime as _real_rt

OK = _real_rt.cudaError_t.cudaSuccess


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _Handle:
    def __init__(self, reserved=b""):
        self.reserved = reserved


class FakeRt:
    """The runtime calls the transport makes, recorded instead of executed."""

    cudaEventDisableTiming = 2
    cudaEventInterprocess = 4
    cudaIpcMemLazyEnablePeerAccess = 1
    cudaIpcMemHandle_t = _Handle
    cudaIpcEventHandle_t = _Handle

    class cudaMemcpyKind:
        cudaMemcpyDeviceToDevice = 3

    def __init__(self, rank, store):
        self.rank, self.store = rank, store
        self.n_events = 0
        self.chain = None
        self.waits = []   # (owner, event index, records seen, chain.calls at the wait, label)
        self.copies = 0
        self.copies2d = 0
        self.label = ""
        self.closed = self.destroyed = self.freed = 0

    def _rec_key(self, ev):
        return f"fake_rec/{ev[0]}/{ev[1]}"

    def cudaMalloc(self, nbytes):
        return OK, 0x10000000 * (self.rank + 1)

    def cudaEventCreateWithFlags(self, flags):
        self.n_events += 1
        return OK, (self.rank, self.n_events - 1)

    def cudaIpcGetMemHandle(self, ptr):
        return OK, _Handle(f"mem{self.rank}".encode())

    def cudaIpcGetEventHandle(self, ev):
        return OK, _Handle(f"{ev[0]}:{ev[1]}".encode())

    def cudaIpcOpenMemHandle(self, h, flags):
        return OK, 0x10000000 * (int(h.reserved.decode()[3:]) + 1)

    def cudaIpcOpenEventHandle(self, h):
        owner, idx = h.reserved.decode().split(":")
        return OK, (int(owner), int(idx))

    def cudaIpcCloseMemHandle(self, ptr):
        self.closed += 1
        return (OK,)

    def cudaEventDestroy(self, ev):
        self.destroyed += 1
        return (OK,)

    def cudaFree(self, ptr):
        self.freed += 1
        return (OK,)

    def cudaEventRecord(self, ev, stream):
        self.store.add(self._rec_key(ev), 1)
        return (OK,)

    def cudaStreamWaitEvent(self, stream, ev, flags):
        seen = self.store.add(self._rec_key(ev), 0)
        self.waits.append((ev[0], ev[1], seen, self.chain.calls, self.label))
        return (OK,)

    def cudaMemcpyAsync(self, dst, src, nbytes, kind, stream):
        self.copies += 1
        return (OK,)

    def cudaMemcpy2DAsync(self, dst, dpitch, src, spitch, width, height, kind, stream):
        assert width <= dpitch and width <= spitch and height >= 1
        self.copies2d += 1
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


def _worker(rank, world, port, root, calls, pieces, n_chunks, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import torch.distributed as dist

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        from fp_emulation import ce_transport as ct

        store = dist.distributed_c10d._get_default_store()
        fake = FakeRt(rank, store)

        class FakeChain(ct.CeChain):
            _rt = fake

            def _device_ctx(self):
                return contextlib.nullcontext()

            def _wrap_buffer(self, ptr, nbytes):
                return None

            def _local_event(self):
                return _LocalEvent()

            def _new_stream(self):
                return _Stream()

            def _current_stream(self):
                return _Stream()

        chain = FakeChain(None, root, None, chunk_bytes=4096, n_chunks=n_chunks, pieces=pieces)
        fake.chain = chain
        main = _Stream()
        # The call sequence of distributed.rowsharded_product_ce, without data.
        for _ in range(calls):
            if rank == root:
                chain.root_begin(main)
                for c in range(n_chunks):
                    chain.root_before_write(c)
                    chain.root_after_write(c)
                chain.root_end()
            else:
                chain.pull()
            for c in range(n_chunks):
                chain.wait_chunk(c, main)
                chain.after_gemm(c, main)
        dist.barrier()
        left = [i for i in range(calls) if store.check([chain._key(rank, i, "A")])]
        q.put((rank, "ok", (chain.pred, chain.succ, fake.waits, fake.copies, left)))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


@pytest.mark.parametrize("world,root", [(2, 0), (3, 1), (4, 2)])
def test_chain_waits_bind_to_the_right_records(world, root):
    calls, pieces, n_chunks = 4, 3, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, root, calls, pieces, n_chunks, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    per_chunk = n_chunks * pieces
    for rank, status, payload in results:
        assert status == "ok", payload
        pred, succ, waits, copies, left = payload
        n_pred = n_succ = n_own = 0
        for owner, _idx, seen, at_call, _label in waits:
            if owner == rank:        # wait_chunk, after this call's records
                assert seen == at_call, (rank, owner, seen, at_call)
                n_own += 1
            elif owner == pred:      # this call's records of the predecessor
                assert seen == at_call + 1, (rank, owner, seen, at_call)
                n_pred += 1
            elif owner == succ:      # the successor's reads of the previous call
                assert seen == at_call, (rank, owner, seen, at_call)
                n_succ += 1
            else:
                raise AssertionError(f"rank {rank} waited on rank {owner}'s event")
        assert n_own == calls * n_chunks
        assert n_pred == (0 if rank == root else calls * per_chunk)
        assert n_succ == (0 if succ is None else (calls - 1) * per_chunk)
        assert copies == (0 if rank == root else calls * per_chunk)
        assert left == [calls - 2, calls - 1], left  # older keys were deleted


# -- the ring: every rank splits a strip, strips go round the ring --------------

# Which call's record each labelled wait must bind to: "war" waits check that a
# reader of the previous call is done (its record of call i-1: i records seen);
# the others wait for data of this call (i+1 records).  GEMM waits come after
# the call counter moved on, so they see exactly `calls` records.
_PREVIOUS_CALL = {"stage war", "split war", "ring war", "gemm"}


def _ring_worker(rank, world, port, root, calls, n_chunks, q, staged=True, pieces=None):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import torch.distributed as dist

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        from fp_emulation import ce_transport as ct
        from fp_emulation.distributed import plan_column_chunks
        from fp_emulation.strips import StripLayout

        store = dist.distributed_c10d._get_default_store()
        fake = FakeRt(rank, store)

        class FakeRing(ct.CeRing):
            _rt = fake

            def _device_ctx(self):
                return contextlib.nullcontext()

            def _wrap_buffer(self, ptr, nbytes):
                return None

            def _local_event(self):
                return _LocalEvent()

            def _new_stream(self):
                return _Stream()

            def _current_stream(self):
                return _Stream()

            def _wait(self, stream, event, what="wait"):
                fake.label = what
                return super()._wait(stream, event, what)

        if staged:
            plan = plan_column_chunks(256 * n_chunks - 100, 256)  # a ragged last chunk
            layout = StripLayout(world, 300, 24, 304, plan)
        else:  # column blocks of 90 columns, strips of 32: chunks of 32, 32 and 26 per rank
            layout = StripLayout.for_blocks(world, 300, 24, 304, 32 * n_chunks - 6, 32)
            plan = layout.plan
        ring = FakeRing(None, root, None, layout, staged=staged, pieces=pieces)
        fake.chain = ring
        splits = []
        main = _Stream()
        for _ in range(calls):
            stage = rank == root and staged
            ring.enqueue(lambda c, ss: splits.append(c), main, 0x1000 if stage else None,
                         256 * n_chunks if stage else None)
            for c in range(len(plan)):
                ring.wait_chunk(c, main)
                ring.after_gemm(c, main)
        dist.barrier()
        left = [i for i in range(calls) if store.check([ring._key(rank, i, "split")])]  # the ring keeps no keys
        q.put((rank, "ok", (ring.pred, ring.succ, fake.waits, fake.copies, fake.copies2d, len(splits), left,
                            len(plan), ring.pieces)))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


@pytest.mark.parametrize("pieces", [None, 4], ids=["default-pieces", "4-pieces"])
@pytest.mark.parametrize("staged", [True, False], ids=["root-staged", "column-sharded"])
@pytest.mark.parametrize("world,root", [(2, 1), (3, 0), (4, 3)])
def test_ring_waits_bind_to_the_right_records(world, root, staged, pieces):
    """Root-staged: the root copies every rank its FP64 strip.  Column-sharded
    (the all-gather product): every rank splits its own block, nothing is staged."""
    calls, n_chunks = 4, 3
    if not staged:
        root = 0
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ring_worker, args=(r, world, port, root, calls, n_chunks, q, staged, pieces))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, status, payload in results:
        assert status == "ok", payload
        pred, succ, waits, copies, copies2d, n_splits, left, nc, P = payload
        counts = {}
        for owner, _idx, seen, at_call, label in waits:
            want = at_call if label in _PREVIOUS_CALL else at_call + 1
            assert seen == want, (rank, owner, label, seen, at_call)
            if label in ("ring", "ring war", "split war"):
                assert owner == (pred if label == "ring" else succ), (rank, owner, label)
            counts[label] = counts.get(label, 0) + 1
        W = world
        assert counts.get("stage war", 0) == (W * nc * (calls - 1) if rank == root and staged else 0)
        assert counts.get("stage", 0) == (nc * calls if staged else 0)
        assert counts.get("split war", 0) == nc * (calls - 1)
        assert counts["ring"] == (W - 1) * nc * calls * P
        assert counts.get("ring war", 0) == (W - 2) * nc * (calls - 1) * P
        assert counts["gemm"] == W * nc * calls
        assert n_splits == nc * calls
        # 2-D copies: the root's FP64 strips (W per chunk) and the ring's residue strips;
        # 1-D copies: the ring's column exponents.
        assert P == (4 if pieces == 4 else 1)
        assert copies2d == (W * nc * calls if rank == root and staged else 0) + (W - 1) * nc * calls * P
        assert copies == (W - 1) * nc * calls
        assert left == [], left


# -- the bounded transport cache: collective least-recently-used eviction --------

def _cache_worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import torch.distributed as dist

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        from fp_emulation import ce_transport as ct
        from fp_emulation import distributed as D

        D.MAX_TRANSPORTS = 2
        store = dist.distributed_c10d._get_default_store()
        fake = FakeRt(rank, store)

        class FakeChain(ct.CeChain):
            _rt = fake

            def _device_ctx(self):
                return contextlib.nullcontext()

            def _wrap_buffer(self, ptr, nbytes):
                return None

            def _local_event(self):
                return _LocalEvent()

            def _new_stream(self):
                return _Stream()

            def _current_stream(self):
                return _Stream()

            def _drain(self):
                pass

        made = {}

        def make(tag):
            def f():
                made[tag] = FakeChain(None, 0, None, chunk_bytes=4096, n_chunks=2, pieces=2)
                return made[tag]
            return f

        main = _Stream()
        for tag in ["a", "b", "a", "c", "d"]:  # a, b; a again (b is now the oldest); c evicts b; d evicts a
            ch = D._cached_transport(None, tag, make(tag))
            fake.chain = ch
            if rank == 0:
                ch.root_begin(main)
                for c in range(2):
                    ch.root_before_write(c)
                    ch.root_after_write(c)
                ch.root_end()
            else:
                ch.pull()
            for c in range(2):
                ch.wait_chunk(c, main)
                ch.after_gemm(c, main)
        dist.barrier()
        released = sorted(t for t, ch in made.items() if ch.ptr is None)
        live = list(D._TRANSPORTS[id(None)].keys())
        keys_left = [t for t in released for i in range(2) if store.check([made[t]._key(rank, i, "A")])]
        q.put((rank, "ok", (released, live, fake.freed, fake.destroyed, fake.closed, keys_left)))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


def test_transport_cache_evicts_the_same_transport_on_every_rank():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_cache_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict((r, (st, pl)) for r, st, pl in (q.get(timeout=180) for _ in range(world)))
    for p in procs:
        p.join(timeout=60)
    for rank, (status, payload) in results.items():
        assert status == "ok", payload
        released, live, freed, destroyed, closed, keys_left = payload
        assert released == ["a", "b"] and live == ["c", "d"]
        assert freed == 2 and keys_left == []
        # Own events: 2 chunks x 2 pieces per transport.  Rank 1 also opened its
        # predecessor's buffer and events in every call; the root opened its
        # successor's events in a's second call only (WAR waits start at call 1).
        if rank == 0:
            assert (destroyed, closed) == (4 + 4 + 4, 0)
        else:
            assert (destroyed, closed) == (2 * (4 + 4), 2)
