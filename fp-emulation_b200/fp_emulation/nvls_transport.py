"""Multi-GPU product over NVLink multicast (NVLS): B's residues are split in
parallel by every GPU and broadcast by the NVSwitch.

Column chunk j of B is cut into one strip per rank.  Per call and chunk:

1. the root copies each rank's FP64 strip of B into that rank's staging slot
   (copy engines, 2-D copies into the peers' memory), then adds 1 to the
   multicast counter ``stage[j]`` (every GPU's copy grows);
2. every rank, once its ``stage[j]`` has reached this call's count, splits its
   strip with ``fpemu_split_mc``: the residues and column exponents are stored
   through the multicast address, so they land in chunk j of every GPU's
   buffer, and each CTA of the split adds 1 to the multicast counter
   ``split[j]`` after its stores;
3. every rank's GEMM on chunk j waits until its ``split[j]`` has grown by all
   ranks' CTA counts, runs on its own copy of the chunk, and then adds 1 to its
   own ``gemm[j]``.

Buffer reuse across calls: a rank splits chunk j of call e only after every
rank's ``gemm[j]`` shows call e-1 done (it polls the peers' counters through
their mappings), and the root overwrites staging slot j only after ``split[j]``
shows call e-1's splits done.

Why: the root alone splitting B costs it 2.7 ms of split work at n = 16384 --
time the power-capped GPU cannot hide under its GEMM -- while here each rank
splits 1/world of B; and multicast stores cost one NVLink egress per byte
where a relay chain or an all-gather of copies costs one per hop.

Safety of the NVLink mappings: every write into another GPU's memory (FP64
strips, multicast residues, multicast counter additions) belongs to a call that
the receiving GPU's own streams wait for before that call ends there, and the
after-GEMM signal is a local addition that peers read.  So once a rank's
streams have drained, nothing writes into its memory until the next call; the
transport drains the device at exit, and on an error while enqueuing it
drains and waits out the peers' bounded waits before raising.
"""
from __future__ import annotations

import atexit
import ctypes
import os
import time

import torch
import torch.distributed as dist
from cuda.bindings import runtime as rt

from fp_emulation import _lib
from fp_emulation.strips import StripLayout, _even_split  # noqa: F401  (re-exported for tests)

NvlsLayout = StripLayout


def _align256(x):
    return (x + 255) // 256 * 256


def _budget_s():
    return max(10, int(os.environ.get("FPEMU_WAIT_BUDGET_MS", "2000"))) / 1000.0


class NvlsTransport:
    """One NVLS channel for a fixed (k, n, n_mod, chunk plan); reused across calls.
    Construction is collective over the group."""

    SPLIT, STAGE, GEMM = 0, 1, 2

    def __init__(self, group, root, device, k, n, n_mod, ld, plan):
        import torch.distributed._symmetric_memory as symm

        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 16:
            raise RuntimeError("the NVLS transport polls at most 16 peers")
        self.root, self.device = root, device
        self.k, self.n, self.n_mod, self.ld, self.plan = k, n, n_mod, ld, plan
        self.lib = _lib.load()
        L = self.layout = NvlsLayout(self.world, k, n_mod, ld, plan)
        self.strips, self.pitch = L.strips, L.pitch
        self.res_bytes, self.chunk_bytes, self.slot_bytes = L.res_bytes, L.chunk_bytes, L.slot_bytes
        self.stage_off, self.cnt_off = L.stage_off, L.cnt_off
        swmax = L.swmax
        self.buf = symm.empty(L.total, dtype=torch.uint8, device=device)
        self.handle = symm.rendezvous(self.buf, group if group is not None else dist.group.WORLD)
        self.mc = int(self.handle.multicast_ptr)
        if self.mc == 0:
            raise RuntimeError("NVLink multicast is not available for this group")
        self.peer = [int(p) for p in self.handle.buffer_ptrs]
        self.local = self.buf.data_ptr()
        self.buf[self.cnt_off:].zero_()
        torch.cuda.synchronize(device)
        dist.barrier(group=group, device_ids=[device.index])
        self.split_stream = torch.cuda.Stream(device)
        self.copy_stream = torch.cuda.Stream(device)
        # GEMMs outrank the splits for SMs that free up: a multicast split is
        # throttled by NVLink and must not hold SMs the next chunk's GEMM needs.
        self.gemm_stream = torch.cuda.Stream(device, priority=-100)
        self.colmax = torch.empty((max(swmax, 1),), dtype=torch.int64, device=device)
        self.signals = [sum(self.lib.fpemu_split_mc_signals(s1 - s0, k) for s0, s1 in row) for row in self.strips]
        self.split_target = [0] * len(plan)
        self.calls = 0
        atexit.register(self.close)

    # -- addresses ------------------------------------------------------------
    def _cnt(self, base, kind, j):
        return base + self.layout.counter(kind, j)

    def chunk_views(self, j):
        return self.layout.chunk_views(self.buf, j)

    # -- enqueue helpers ------------------------------------------------------
    def _wait(self, addrs, target, where, stream):
        arr = (ctypes.c_uint64 * len(addrs))(*addrs)
        _lib.check(self.lib.fpemu_wait_counters(arr, len(addrs), target, where, stream.cuda_stream),
                   "wait_counters")

    def _signal(self, addr, multicast, stream):
        _lib.check(self.lib.fpemu_signal_counter(addr, 1 if multicast else 0, stream.cuda_stream), "signal_counter")

    def _stage_copies(self, B, e, main):
        cs = self.copy_stream
        cs.wait_stream(main)
        B.record_stream(cs)
        ldb = B.stride(0)
        for j, (c0, c1) in enumerate(self.plan):
            if e > 1:  # every rank's split of call e-1 has read its slot j
                self._wait([self._cnt(self.local, self.SPLIT, j)], self.split_target[j], 1, cs)
            dst_slot = self.stage_off + j * self.slot_bytes
            for q, (s0, s1) in enumerate(self.strips[j]):
                w = s1 - s0
                if w == 0:
                    continue
                err = rt.cudaMemcpy2DAsync(self.peer[q] + dst_slot, self.pitch * 8,
                                           B.data_ptr() + (c0 + s0) * 8, ldb * 8, w * 8, self.k,
                                           rt.cudaMemcpyKind.cudaMemcpyDeviceToDevice, cs.cuda_stream)
                if err[0] != rt.cudaError_t.cudaSuccess:
                    raise RuntimeError(f"staging copy failed: {err[0]}")
            self._signal(self._cnt(self.mc, self.STAGE, j), True, cs)

    def _splits(self, bits, e):
        ss = self.split_stream
        r = self.rank
        for j, (c0, c1) in enumerate(self.plan):
            w = c1 - c0
            s0, s1 = self.strips[j][r]
            self._wait([self._cnt(self.local, self.STAGE, j)], e, 2, ss)
            if e > 1:  # every GPU's GEMM of call e-1 is done with chunk j
                self._wait([self._cnt(p, self.GEMM, j) for p in self.peer], e - 1, 3, ss)
            if s1 == s0:
                continue
            base = self.mc + j * self.chunk_bytes
            st = self.lib.fpemu_split_mc(s1 - s0, self.k, self.local + self.stage_off + j * self.slot_bytes, 1,
                                         self.pitch, bits, self.n_mod, base + s0 * self.ld, self.ld, w * self.ld,
                                         base + self.res_bytes + 4 * s0, self.colmax.data_ptr(),
                                         self._cnt(self.mc, self.SPLIT, j), ss.cuda_stream)
            _lib.check(st, "split_mc")

    # -- one collective product ----------------------------------------------
    def product(self, A_local, B, ops, bits):
        """C_local [m, n] = A_local @ B; B is read on the root only."""
        e = self.calls + 1
        main = torch.cuda.current_stream(self.device)
        try:
            if self.rank == self.root:
                if B.stride(1) != 1:
                    B = B.contiguous()
                self._stage_copies(B, e, main)
            self._splits(bits, e)
            for j in range(len(self.plan)):
                self.split_target[j] += self.signals[j]
            m = A_local.shape[0]
            C = torch.empty((m, self.n), dtype=torch.float64, device=self.device)
            gs = self.gemm_stream
            gs.wait_stream(main)
            A_local.record_stream(gs)
            C.record_stream(gs)
            with torch.cuda.stream(gs):
                a_res = ops.empty_res(self.n_mod, m, self.ld)
                row_exp = ops.empty_exps(m)
                ops.split(A_local, bits, self.n_mod, a_res, row_exp)
                for j, (c0, c1) in enumerate(self.plan):
                    res, exps = self.chunk_views(j)
                    self._wait([self._cnt(self.local, self.SPLIT, j)], self.split_target[j], 4, gs)
                    if m and c1 > c0:
                        ops.gemm_crt(a_res, row_exp, res, exps, bits, C, c0, c1, self.k)
                    self._signal(self._cnt(self.local, self.GEMM, j), False, gs)
            main.wait_stream(gs)
            self.calls = e
            return C
        except BaseException:
            # Let this GPU's queued work and the peers' bounded waits run out
            # before this process can go away with its memory still mapped.
            torch.cuda.synchronize(self.device)
            time.sleep(_budget_s() + 1.0)
            raise

    def close(self):
        try:
            torch.cuda.synchronize(self.device)
        except Exception:
            pass

    def release(self, barrier):
        """Drop the symmetric buffer.  Collective (every rank releases the same
        transport in the same call): this device drains, the group meets -- after
        which no rank stores into another's copy -- then the references go."""
        torch.cuda.synchronize(self.device)
        barrier()
        self.buf = self.handle = self.colmax = None
        atexit.unregister(self.close)
