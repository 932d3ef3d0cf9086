"""Column strips of B's chunks and the byte layout of the per-GPU buffer that
holds them, for the transport in which every GPU splits one strip of each
chunk (the copy-engine ring, ce_transport.CeRing)."""
from __future__ import annotations

import torch


def _align256(x):
    return (x + 255) // 256 * 256


def _even_split(w, parts, i):
    """Columns [s0, s1) of part i when w columns are cut into `parts` near-equal strips."""
    base, extra = divmod(w, parts)
    s0 = i * base + min(i, extra)
    return s0, s0 + base + (1 if i < extra else 0)


class StripLayout:
    """Byte layout of a GPU's buffer for one (world, k, n_mod, ld, plan):
    [chunk 0 .. chunk nc-1 | staging slot 0 .. nc-1].

    chunk j: int8 residues [n_mod][w_j][ld] (plane stride w_j * ld), then the
    w_j int32 column exponents at res_bytes; strip q of chunk j is columns
    strips[j][q] of the chunk.  Staging slot j: rank's FP64 strip, k rows of
    `pitch` doubles (pitch >= 2 keeps the split's K stride non-unit)."""

    def __init__(self, world, k, n_mod, ld, plan, strips=None, staging=True):
        self.world, self.k, self.n_mod, self.ld, self.plan = world, k, n_mod, ld, plan
        nc = len(plan)
        self.strips = strips or [[_even_split(c1 - c0, world, q) for q in range(world)] for c0, c1 in plan]
        wmax = max(c1 - c0 for c0, c1 in plan)
        swmax = max(s1 - s0 for row in self.strips for s0, s1 in row)
        self.swmax = swmax
        self.pitch = max(swmax, 2)
        self.res_bytes = _align256(n_mod * wmax * ld)
        self.chunk_bytes = self.res_bytes + _align256(wmax * 4)
        self.slot_bytes = _align256(k * self.pitch * 8) if staging else 0
        self.stage_off = nc * self.chunk_bytes
        self.total = self.stage_off + nc * self.slot_bytes
        self.block_cols = None  # set by for_blocks
        self.block_off = None

    @classmethod
    def for_blocks(cls, world, k, n_mod, ld, block_cols, strip_cols):
        """Layout for B column-sharded in equal blocks of `block_cols` columns
        (GPU q holds columns [q*block_cols, (q+1)*block_cols) of B).  Chunk c
        gathers columns [c*strip_cols, c*strip_cols + w_c) of every GPU's block,
        w_c = min(strip_cols, block_cols - c*strip_cols): strip q of chunk c is
        GPU q's piece, columns [q*w_c, (q+1)*w_c) of the chunk.  No staging slots
        (every GPU splits its own block).  `plan` lists the chunks' column ranges
        as if the chunks were laid side by side; block_off[c] = c*strip_cols is
        where chunk c starts inside each block."""
        if block_cols < 1 or strip_cols < 1:
            raise ValueError("block and strip widths must be positive")
        plan, strips, offs, off = [], [], [], 0
        for c0 in range(0, block_cols, strip_cols):
            w = min(strip_cols, block_cols - c0)
            plan.append((off, off + world * w))
            strips.append([(q * w, (q + 1) * w) for q in range(world)])
            offs.append(c0)
            off += world * w
        L = cls(world, k, n_mod, ld, plan, strips=strips, staging=False)
        L.block_cols = block_cols
        L.block_off = offs
        return L

    def residue_span(self, j, q):
        """[first, last] byte offsets the split of strip q of chunk j writes
        (residues), and the same for its exponents; None for an empty strip."""
        c0, c1 = self.plan[j]
        w = c1 - c0
        s0, s1 = self.strips[j][q]
        if s1 == s0:
            return None
        base = j * self.chunk_bytes
        res = (base + s0 * self.ld, base + (self.n_mod - 1) * w * self.ld + (s1 - 1) * self.ld + self.ld - 1)
        exps = (base + self.res_bytes + 4 * s0, base + self.res_bytes + 4 * s1 - 1)
        return res, exps

    def staging_span(self, j, q):
        """[first, last] byte offsets the 2-D copy of strip q fills in slot j."""
        s0, s1 = self.strips[j][q]
        if s1 == s0:
            return None
        base = self.stage_off + j * self.slot_bytes
        return base, base + (self.k - 1) * self.pitch * 8 + (s1 - s0) * 8 - 1

    # -- typed views of a GPU's buffer (a flat uint8 tensor laid out as above) --
    def chunk_views(self, buf, j):
        """(residues int8 [n_mod][w_j][ld], column exponents int32 [w_j]) of chunk j."""
        c0, c1 = self.plan[j]
        w = c1 - c0
        blk = buf[j * self.chunk_bytes:(j + 1) * self.chunk_bytes]
        return (blk[: self.n_mod * w * self.ld].view(self.n_mod, w, self.ld),
                blk[self.res_bytes: self.res_bytes + 4 * w].view(torch.int32))

    def staging_strip(self, buf, j, q):
        """Strip q of chunk j as the split reads it from staging slot j: float64
        [w_q, k] with strides (1, pitch) -- the strip's columns of B as rows, K
        strided (the 2-D copy wrote k rows of `pitch` doubles)."""
        s0, s1 = self.strips[j][q]
        off = self.stage_off + j * self.slot_bytes
        slot = buf[off: off + 8 * self.k * self.pitch]
        return slot.view(torch.float64).view(self.k, self.pitch)[:, : s1 - s0].T

