"""Multi-GPU row-sharded Ozaki-II product: C[rows of this rank] = A_local @ B.

The reference has no multi-GPU code; this is the build's one exchange step.
A is split by row blocks (each rank holds its own rows; their exponents are
per row, so no communication), and C is sharded the same way.  B is needed
whole everywhere: the root rank splits it once into int8 residue planes plus
column exponents and broadcasts them with NCCL over NVLink.  K is never split,
so there is no reduction collective.

The broadcast runs on NCCL's stream while this rank splits its own A rows on
the compute stream; the fused GEMM + CRT kernel starts when both are done.
One process per GPU (torch.distributed, backend "nccl"; "gloo" works for the
host-side logic in tests).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from fp_emulation import _lib
from fp_emulation.ozaki import (_PRECISION_BITS, _after_call, _n_moduli, _require_cuda, _res_ld,
                                _split, _stream)


def shard_rows(m: int, world: int, rank: int):
    """Row range [r0, r1) of rank `rank` when m rows are split as evenly as possible."""
    base, extra = divmod(m, world)
    r0 = rank * base + min(rank, extra)
    return r0, r0 + base + (1 if rank < extra else 0)


def broadcast_b_residues(B, n: int, k: int, bits: int, n_mod: int, root: int = 0, group=None,
                         device=None, async_op: bool = False):
    """Split B ([k, n], on `root`) into residues and broadcast them.

    Returns (b_res int8 [n_mod, n, res_ld], col_exp int32 [n], work) where `work`
    is the pending broadcast handle when async_op=True (wait() on it before use).
    Non-root ranks pass B=None.
    """
    rank = dist.get_rank(group)
    dev = device if device is not None else (B.device if B is not None else torch.device("cuda"))
    if rank == root:
        _require_cuda(B)
        b_res, col_exp = _split(B.T, bits, n_mod)
    else:
        b_res = torch.empty((n_mod, n, _res_ld(k)), dtype=torch.int8, device=dev)
        col_exp = torch.empty((n,), dtype=torch.int32, device=dev)
    w1 = dist.broadcast(b_res, src=root, group=group, async_op=True)
    w2 = dist.broadcast(col_exp, src=root, group=group, async_op=True)

    class _Both:
        def wait(self):
            w1.wait()
            w2.wait()

    work = _Both()
    if not async_op:
        work.wait()
        return b_res, col_exp, None
    return b_res, col_exp, work


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
    m, k = A_local.shape
    rank = dist.get_rank(group)
    if rank == root:
        if B is None or B.shape[0] != k:
            raise RuntimeError("root must pass B with B.shape[0] == A_local.shape[1]")
        B = B.double()
        n = B.shape[1]
    if n is None:
        raise RuntimeError("non-root ranks must pass n (B's column count)")
    n_mod = _n_moduli(k, bits)
    b_res, col_exp, work = broadcast_b_residues(B, n, k, bits, n_mod, root, group, dev, async_op=True)
    a_res, row_exp = _split(A_local, bits, n_mod)   # overlaps the broadcast
    work.wait()
    C = torch.empty((m, n), dtype=torch.float64, device=dev)
    if m and n:
        lib = _lib.load()
        nbytes = lib.fpemu_gemm_workspace_size(m, n, n_mod)
        ws = torch.empty((max(nbytes, 256),), dtype=torch.uint8, device=dev)
        with torch.cuda.device(dev):
            st = lib.fpemu_gemm_crt(m, n, k, n_mod, a_res.data_ptr(), b_res.data_ptr(), _res_ld(k),
                                    row_exp.data_ptr(), col_exp.data_ptr(), bits, C.data_ptr(), n,
                                    ws.data_ptr(), ws.numel(), _stream(dev))
        _lib.check(st, "ozaki2_int8_matmul_rowsharded")
        _after_call("ozaki2_int8_matmul_rowsharded")
    return C if orig == torch.float64 else C.to(orig)
