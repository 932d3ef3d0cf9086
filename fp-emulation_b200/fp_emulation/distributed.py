"""Multi-GPU row-sharded Ozaki-II product: C[rows of this rank] = A_local @ B.

The reference has no multi-GPU code; this is the build's one exchange step.
A is split by row blocks: each rank holds its own rows, whose exponents are
per row, so splitting them needs no communication, and C is sharded the same
way.  B, held by one root rank, is needed whole everywhere, as int8 residue
planes plus column exponents.  K is never split, so there is no reduction
collective.  One process per GPU (torch.distributed).

The product is pipelined by column chunks of B: every rank runs the fused GEMM
+ CRT for chunk c (its rows x the chunk's columns of C) as soon as chunk c's
residues are in its memory, while later chunks are in flight.  How they get
there is the transport (TRANSPORT below): a copy-engine chain through CUDA IPC
(default), a copy-engine ring of per-rank strips, or NCCL broadcasts.

The NCCL pipeline is written against a small backend (`_GpuOps`) so that it
can be exercised with CPU ranks over gloo in tests.
"""
from __future__ import annotations

import os
from collections import OrderedDict
from dataclasses import dataclass

import torch
import torch.distributed as dist

from fp_emulation import _lib
from fp_emulation.ozaki import (_PRECISION_BITS, _after_call, _n_moduli, _require_cuda, _res_ld,
                                _stream)

# Column chunk width of the pipelined broadcast (a multiple of the GEMM's 256-wide tiles).
CHUNK_COLS = int(os.environ.get("FPEMU_CHUNK_COLS", "2048"))
# SMs left to NCCL while a chunk's GEMM runs.
COMM_SMS = int(os.environ.get("FPEMU_COMM_SMS", "16"))
# What the root broadcasts: "residues" (B's int8 residue planes, n_mod bytes per
# element, the default) or "fp64" (B itself, 8 bytes per element; every rank then
# splits the chunk locally -- less NVLink traffic for more split work per rank).
BCAST_MODE = os.environ.get("FPEMU_BCAST", "residues")
# How B's residues reach every rank:
#  "ce" (default): the root splits B, copy engines relay the chunks along a chain
#         of ranks through CUDA IPC (ce_transport.py);
#  "ce-ring": every rank splits a strip of each chunk (FP64 strips copied from the
#         root), the residue strips go round a ring by the copy engines, chunk
#         after chunk (ce_transport.CeRing);
#  "nccl": the root splits B, NCCL broadcast kernels move the chunks.
TRANSPORT = os.environ.get("FPEMU_TRANSPORT", "ce")


def shard_rows(m: int, world: int, rank: int):
    """Row range [r0, r1) of rank `rank` when m rows are split as evenly as possible."""
    base, extra = divmod(m, world)
    r0 = rank * base + min(rank, extra)
    return r0, r0 + base + (1 if rank < extra else 0)


def plan_column_chunks(n: int, chunk_cols: int = CHUNK_COLS, align: int = 256):
    """Column ranges [c0, c1) covering [0, n); every chunk but the last is a
    multiple of `align` wide."""
    w = max(align, (chunk_cols // align) * align)
    return [(c0, min(n, c0 + w)) for c0 in range(0, n, w)] or [(0, 0)]


@dataclass
class _Chunk:
    c0: int
    c1: int
    res: torch.Tensor      # int8 [n_mod, c1 - c0, ld] (contiguous: one broadcast)
    work: object = None
    fp64: torch.Tensor = None  # mode "fp64": the chunk of B, [k, c1 - c0]


class _GpuOps:
    """The product backend: libfpemu through the C ABI on the current stream."""

    def __init__(self, device, timing=None, comm_sms=None):
        self.device = device
        self.lib = _lib.load()
        props = torch.cuda.get_device_properties(device)
        spare = COMM_SMS if comm_sms is None else comm_sms
        self.max_ctas = 0 if spare <= 0 else max(2, props.multi_processor_count - spare)
        self.timing = timing  # optional list collecting (start, end, int8_ops) per GEMM launch

    def empty_res(self, n_mod, rows, ld):
        return torch.empty((n_mod, rows, ld), dtype=torch.int8, device=self.device)

    def empty_exps(self, rows):
        return torch.empty((rows,), dtype=torch.int32, device=self.device)

    def split(self, X, bits, n_mod, res, exps):
        """Residues of the rows of X [rows, k] into res [n_mod, rows, ld], exponents into exps."""
        rows, k = X.shape
        ld = res.shape[2]
        colmax = torch.empty((max(rows, 1),), dtype=torch.int64, device=self.device) if X.stride(1) != 1 else None
        st = self.lib.fpemu_split(rows, k, X.data_ptr(), X.stride(0), X.stride(1), bits, n_mod, res.data_ptr(),
                                  ld, res.stride(0), exps.data_ptr(),
                                  None if colmax is None else colmax.data_ptr(), _stream(self.device))
        _lib.check(st, "split")

    def gemm_crt(self, a_res, re, b_res, ce_chunk, bits, C, c0, c1, k):
        """C[:, c0:c1] from A's residues and one column chunk of B's (ce_chunk: that
        chunk's column exponents)."""
        n_mod, m, ld = a_res.shape
        w = c1 - c0
        nbytes = self.lib.fpemu_gemm_workspace_size(m, w, n_mod)
        ws = torch.empty((max(nbytes, 256),), dtype=torch.uint8, device=self.device)
        Cv = C[:, c0:c1]
        if self.timing is not None:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        st = self.lib.fpemu_gemm_crt(m, w, k, n_mod, a_res.data_ptr(), b_res.data_ptr(), ld, b_res.stride(0),
                                     re.data_ptr(), ce_chunk.data_ptr(), bits, Cv.data_ptr(), C.stride(0),
                                     self.max_ctas, ws.data_ptr(), ws.numel(), _stream(self.device))
        _lib.check(st, "gemm_crt")
        if self.timing is not None:
            ev[1].record()
            self.timing.append((ev[0], ev[1], 2.0 * m * w * k * n_mod))


    def gemm_crt_segmented(self, a_res, re, b_res, ce_chunk, bits, C, col_off, seg, seg_stride, k):
        """C[:, cols] for one all-gathered chunk: chunk column j goes to C column
        col_off + (j // seg) * seg_stride + j % seg."""
        n_mod, m, ld = a_res.shape
        w = b_res.shape[1]
        nbytes = self.lib.fpemu_gemm_workspace_size(m, w, n_mod)
        ws = torch.empty((max(nbytes, 256),), dtype=torch.uint8, device=self.device)
        if self.timing is not None:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        st = self.lib.fpemu_gemm_crt_segmented(m, w, k, n_mod, a_res.data_ptr(), b_res.data_ptr(), ld,
                                               b_res.stride(0), re.data_ptr(), ce_chunk.data_ptr(), bits,
                                               C.data_ptr() + 8 * col_off, C.stride(0), seg, seg_stride,
                                               self.max_ctas, ws.data_ptr(), ws.numel(), _stream(self.device))
        _lib.check(st, "gemm_crt_segmented")
        if self.timing is not None:
            ev[1].record()
            self.timing.append((ev[0], ev[1], 2.0 * m * w * k * n_mod))


def rowsharded_product(A_local, B, n, k, bits, n_mod, ops, root=0, group=None, chunk_cols=CHUNK_COLS,
                       mode=None):
    """The pipeline: chunked split/broadcast of B's residues (or of B itself,
    mode "fp64"), split of A's rows, one fused GEMM per chunk.  Returns C_local
    [m_local, n] (float64)."""
    mode = mode or BCAST_MODE
    if mode not in ("residues", "fp64"):
        raise ValueError(f"broadcast mode {mode!r}")
    rank = dist.get_rank(group)
    m = A_local.shape[0]
    ld = _res_ld(k)
    col_exp = ops.empty_exps(n)
    chunks = []
    for c0, c1 in plan_column_chunks(n, chunk_cols):
        ch = _Chunk(c0, c1, ops.empty_res(n_mod, c1 - c0, ld))
        if mode == "residues":
            if rank == root:
                ops.split(B[:, c0:c1].T, bits, n_mod, ch.res, col_exp[c0:c1])
            ch.work = dist.broadcast(ch.res, src=root, group=group, async_op=True)
        else:
            ch.fp64 = (B[:, c0:c1].contiguous() if rank == root
                       else torch.empty((k, c1 - c0), dtype=torch.float64, device=A_local.device))
            ch.work = dist.broadcast(ch.fp64, src=root, group=group, async_op=True)
        chunks.append(ch)
    exp_work = (dist.broadcast(col_exp, src=root, group=group, async_op=True) if mode == "residues" else None)
    a_res = ops.empty_res(n_mod, m, ld)
    row_exp = ops.empty_exps(m)
    ops.split(A_local, bits, n_mod, a_res, row_exp)   # overlaps the broadcasts
    C = torch.empty((m, n), dtype=torch.float64, device=A_local.device)
    if exp_work is not None:
        exp_work.wait()
    if mode == "fp64":
        # Split every chunk as it lands (short kernels that interleave with NCCL's
        # CTAs), then run the GEMMs on all SMs.
        for ch in chunks:
            ch.work.wait()
            ops.split(ch.fp64.T, bits, n_mod, ch.res, col_exp[ch.c0:ch.c1])
    for ch in chunks:
        if mode == "residues":
            ch.work.wait()                              # this chunk has arrived
        if m and ch.c1 > ch.c0:
            ops.gemm_crt(a_res, row_exp, ch.res, col_exp[ch.c0:ch.c1], bits, C, ch.c0, ch.c1, k)
    return C


# Transports hold large device buffers (B's residues for every chunk of one
# column layout), so each process group keeps at most MAX_TRANSPORTS of them,
# the least recently used evicted first.  The products are collective calls made
# in the same order on every rank, so every rank evicts the same transport in the
# same call, and the release can meet the group.
MAX_TRANSPORTS = int(os.environ.get("FPEMU_MAX_TRANSPORTS", "4"))
_TRANSPORTS = {}  # id(group) -> OrderedDict(key -> transport), oldest first


def _group_barrier(group, device):
    if device is not None and dist.get_backend(group) == "nccl":
        dist.barrier(group=group, device_ids=[device.index])
    else:
        dist.barrier(group=group)


def _cached_transport(group, key, make):
    """The transport for `key` (made by `make()` on a miss), most recent first."""
    cache = _TRANSPORTS.setdefault(id(group), OrderedDict())
    tr = cache.pop(key, None)
    if tr is None:
        while cache and len(cache) >= max(1, MAX_TRANSPORTS):
            _, old = cache.popitem(last=False)
            old.release(lambda: _group_barrier(group, getattr(old, "device", None)))
        tr = make()
    cache[key] = tr
    return tr


def _align256(x):
    return (x + 255) // 256 * 256


def rowsharded_product_ring(A_local, B, n, k, bits, n_mod, ops, root=0, group=None, chunk_cols=CHUNK_COLS):
    """Same product through the copy-engine ring (ce_transport.CeRing): the root
    copies each rank its FP64 strip of every chunk, every rank splits its strip,
    and the residue strips go round the ring by the copy engines, chunk after
    chunk (FPEMU_TRANSPORT=ce-ring)."""
    from fp_emulation.ce_transport import CeRing
    from fp_emulation.strips import StripLayout

    rank = dist.get_rank(group)
    dev = A_local.device
    m = A_local.shape[0]
    ld = _res_ld(k)
    plan = plan_column_chunks(n, chunk_cols)
    key = ("ce-ring", root, dev.index, k, n, n_mod, tuple(plan))
    tr = _cached_transport(group, key, lambda: CeRing(group, root, dev,
                                                      StripLayout(dist.get_world_size(group), k, n_mod, ld, plan)))
    L = tr.layout
    stream = torch.cuda.current_stream(dev)

    def views(c):
        return L.chunk_views(tr.buf, c)

    Bc = None
    if rank == root:
        Bc = B if B.stride(1) == 1 else B.contiguous()
        Bc.record_stream(tr.copy_stream)

    def split_fn(c, ss):
        s0, s1 = L.strips[c][rank]
        if s1 == s0:
            return
        res, exps = views(c)
        X = L.staging_strip(tr.buf, c, rank)  # the strip's columns as rows, K strided
        with torch.cuda.stream(ss):
            ops.split(X, bits, n_mod, res[:, s0:s1, :], exps[s0:s1])

    tr.enqueue(split_fn, stream, Bc.data_ptr() if Bc is not None else None, Bc.stride(0) if Bc is not None else None)
    a_res = ops.empty_res(n_mod, m, ld)
    row_exp = ops.empty_exps(m)
    ops.split(A_local, bits, n_mod, a_res, row_exp)
    C = torch.empty((m, n), dtype=torch.float64, device=dev)
    for c, (c0, c1) in enumerate(plan):
        res, exps = views(c)
        tr.wait_chunk(c, stream)
        if m and c1 > c0:
            ops.gemm_crt(a_res, row_exp, res, exps, bits, C, c0, c1, k)
        tr.after_gemm(c, stream)
    return C


def rowsharded_product_auto(A_local, B, n, k, bits, n_mod, ops, root=0, group=None, transport=None):
    """The product through the configured transport."""
    kind = transport or TRANSPORT
    if BCAST_MODE != "residues" or kind == "nccl":
        return rowsharded_product(A_local, B, n, k, bits, n_mod, ops, root, group)
    if kind == "ce-ring":
        return rowsharded_product_ring(A_local, B, n, k, bits, n_mod, ops, root, group)
    if kind != "ce":
        raise ValueError(f"unknown transport {kind!r} (ce, ce-ring, nccl)")
    return rowsharded_product_ce(A_local, B, n, k, bits, n_mod, ops, root, group, transport=kind)


def rowsharded_product_ce(A_local, B, n, k, bits, n_mod, ops, root=0, group=None, chunk_cols=CHUNK_COLS,
                          transport=None):
    """Same product, B's residues moved by the copy engines (ce_transport.py).

    The root splits each column chunk straight into its shared buffer on a side
    stream, so the splits run on the SMs the wave-balanced GEMM grid leaves free
    while the root's GEMMs start on the first chunk; every other rank pulls the
    chunks over NVLink and starts its GEMM on chunk c when chunk c has landed.
    No SMs are spent on the transfer."""
    from fp_emulation.ce_transport import TRANSPORTS

    kind = transport or TRANSPORT
    rank = dist.get_rank(group)
    dev = A_local.device
    m = A_local.shape[0]
    ld = _res_ld(k)
    plan = plan_column_chunks(n, chunk_cols)
    wmax = max(c1 - c0 for c0, c1 in plan)
    res_bytes = _align256(n_mod * wmax * ld)
    chunk_bytes = res_bytes + _align256(wmax * 4)
    key = (kind, root, dev.index, chunk_bytes, len(plan))
    tr = _cached_transport(group, key, lambda: TRANSPORTS[kind](group, root, dev, chunk_bytes, len(plan)))
    stream = torch.cuda.current_stream(dev)
    views = []
    for c, (c0, c1) in enumerate(plan):
        w = c1 - c0
        blk = tr.chunk_view(c)
        views.append((c0, c1, blk[: n_mod * w * ld].view(n_mod, w, ld),
                      blk[res_bytes: res_bytes + 4 * w].view(torch.int32)))
    if rank == root:
        tr.root_begin(stream)
        ss = tr.split_stream
        if ss is not stream:
            B.record_stream(ss)
        with torch.cuda.stream(ss):
            for c, (c0, c1, res, exps) in enumerate(views):
                tr.root_before_write(c)
                ops.split(B[:, c0:c1].T, bits, n_mod, res, exps)
                tr.root_after_write(c)
        tr.root_end()
    else:
        tr.pull()
    a_res = ops.empty_res(n_mod, m, ld)
    row_exp = ops.empty_exps(m)
    ops.split(A_local, bits, n_mod, a_res, row_exp)
    C = torch.empty((m, n), dtype=torch.float64, device=dev)
    for c, (c0, c1, res, exps) in enumerate(views):
        tr.wait_chunk(c, stream)
        if m and c1 > c0:
            ops.gemm_crt(a_res, row_exp, res, exps, bits, C, c0, c1, k)
        tr.after_gemm(c, stream)
    return C


def allgather_strip_cols(world, chunk_cols=CHUNK_COLS):
    """Columns each GPU contributes to one chunk of the all-gathered product
    (CHUNK_COLS across the group, a multiple of 16)."""
    return max(16, (chunk_cols // world) // 16 * 16)


def rowsharded_product_allgather(A_local, B_local, k, bits, n_mod, ops, group=None, strip_cols=None):
    """C_local = A_local @ B with B column-sharded: this rank holds columns
    [q*nb, (q+1)*nb) of B as B_local [k, nb].  Chunk c gathers strip
    [c*sw, c*sw + w_c) of every rank's block; each rank splits its own strips
    (no root), the residue strips go round the copy-engine ring (CeRing,
    unstaged), and the GEMM of chunk c writes each strip's columns to their
    place in C through the segmented epilogue."""
    from fp_emulation.ce_transport import CeRing
    from fp_emulation.strips import StripLayout

    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    dev = A_local.device
    m = A_local.shape[0]
    nb = B_local.shape[1]
    ld = _res_ld(k)
    sw = strip_cols or allgather_strip_cols(world)
    key = ("allgather", dev.index, k, nb, n_mod, sw)

    def make():
        # Collective: every rank must hold a block of the same shape.
        shapes = [None] * world
        dist.all_gather_object(shapes, (k, nb, n_mod), group=group)
        if any(x != shapes[0] for x in shapes):
            raise RuntimeError(f"column-sharded B: every rank needs a [k, nb] block of one shape, got {shapes}")
        return CeRing(group, 0, dev, StripLayout.for_blocks(world, k, n_mod, ld, nb, sw), staged=False)

    tr = _cached_transport(group, key, make)
    L = tr.layout
    stream = torch.cuda.current_stream(dev)
    B_local.record_stream(tr.split_stream)

    def split_fn(c, ss):
        s0, s1 = L.strips[c][rank]
        res, exps = L.chunk_views(tr.buf, c)
        X = B_local[:, L.block_off[c]: L.block_off[c] + (s1 - s0)].T  # the strip's columns as rows, K strided
        with torch.cuda.stream(ss):
            ops.split(X, bits, n_mod, res[:, s0:s1, :], exps[s0:s1])

    tr.enqueue(split_fn, stream)
    a_res = ops.empty_res(n_mod, m, ld)
    row_exp = ops.empty_exps(m)
    ops.split(A_local, bits, n_mod, a_res, row_exp)
    C = torch.empty((m, world * nb), dtype=torch.float64, device=dev)
    for c, (c0, c1) in enumerate(L.plan):
        res, exps = L.chunk_views(tr.buf, c)
        tr.wait_chunk(c, stream)
        if m and c1 > c0:
            ops.gemm_crt_segmented(a_res, row_exp, res, exps, bits, C, L.block_off[c], L.strips[c][0][1], nb, k)
        tr.after_gemm(c, stream)
    return C


def ozaki2_int8_matmul_allgather(A_local, B_local, group=None):
    """C_local = A_local @ B with A row-sharded and B column-sharded across the
    ranks of `group`: rank q passes its rows of A and its block of columns
    [q*nb, (q+1)*nb) of B (every rank the same nb), and gets its rows of C over
    all world*nb columns (float64, or A's dtype), bit-identical to the
    single-GPU product.  B's residues are all-gathered over NVLink by the copy
    engines, pipelined with the GEMMs.  Called collectively, in the same order on
    every rank.  Not in the reference, which has no multi-GPU path."""
    bits = _PRECISION_BITS.get(A_local.dtype)
    if bits is None:
        raise TypeError(f"unsupported dtype {A_local.dtype}")
    dev = _require_cuda(A_local, B_local)
    orig = A_local.dtype
    A_local, B_local = A_local.double(), B_local.double()
    k = A_local.shape[1]
    if B_local.dim() != 2 or B_local.shape[0] != k:
        raise RuntimeError(f"B_local must be [k, nb] with k = {k}, got {tuple(B_local.shape)}")
    if k == 0:
        raise RuntimeError("inner dimension k must be non-zero")
    n_mod = _n_moduli(k, bits)
    with torch.cuda.device(dev):
        if dist.get_world_size(group) == 1:
            from fp_emulation.ozaki import _ozaki2_forward

            C = _ozaki2_forward(A_local, B_local, n_mod=n_mod)
        else:
            C = rowsharded_product_allgather(A_local, B_local, k, bits, n_mod, _GpuOps(dev, comm_sms=0), group)
    _after_call("ozaki2_int8_matmul_allgather", dev)
    return C if orig == torch.float64 else C.to(orig)


def ozaki2_int8_matmul_rowsharded(A_local, B, n: int | None = None, root: int = 0, group=None):
    """C_local = A_local @ B with A row-sharded across the ranks of `group` and B
    held by `root` (other ranks pass B=None and its column count `n`).

    Every rank gets its own rows of C (float64, or A's dtype).  All ranks call
    this collectively, in the same order.
    """
    bits = _PRECISION_BITS.get(A_local.dtype)
    if bits is None:
        raise TypeError(f"unsupported dtype {A_local.dtype}")
    dev = _require_cuda(A_local)
    orig = A_local.dtype
    A_local = A_local.double()
    k = A_local.shape[1]
    if dist.get_rank(group) == root:
        if B is None or B.dim() != 2 or B.shape[0] != k:
            raise RuntimeError("root must pass B with B.shape[0] == A_local.shape[1]")
        _require_cuda(B)
        B = B.double()
        n = B.shape[1]
    if n is None:
        raise RuntimeError("non-root ranks must pass n (B's column count)")
    if k == 0:
        raise RuntimeError("inner dimension k must be non-zero")
    n_mod = _n_moduli(k, bits)
    with torch.cuda.device(dev):
        if dist.get_world_size(group) == 1:
            from fp_emulation.ozaki import _ozaki2_forward

            C = _ozaki2_forward(A_local, B, n_mod=n_mod)
        else:
            ops = _GpuOps(dev, comm_sms=None if TRANSPORT == "nccl" or BCAST_MODE != "residues" else 0)
            C = rowsharded_product_auto(A_local, B, n, k, bits, n_mod, ops, root, group)
    _after_call("ozaki2_int8_matmul_rowsharded", dev)
    return C if orig == torch.float64 else C.to(orig)
