"""Index arithmetic of the multi-GPU transports, checked on the CPU: every
byte range a kernel or a copy writes lies inside its own region of the
shared buffer, regions do not overlap, and the strips and pieces partition
their chunks exactly (no GPU needed)."""
from __future__ import annotations

import itertools

import pytest

from fp_emulation.distributed import plan_column_chunks
from fp_emulation.strips import StripLayout, _even_split
from fp_emulation.ozaki import _res_ld


@pytest.mark.parametrize("w,parts", [(0, 3), (1, 8), (7, 8), (256, 8), (476, 8), (2048, 8), (2047, 3), (5, 2)])
def test_even_split_partitions(w, parts):
    spans = [_even_split(w, parts, i) for i in range(parts)]
    assert spans[0][0] == 0 and spans[-1][1] == w
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 == b0 and a0 <= a1
    sizes = [s1 - s0 for s0, s1 in spans]
    assert max(sizes) - min(sizes) <= 1


CASES = [(2, 700, 24, 1500, 512), (8, 700, 24, 1500, 512), (3, 129, 24, 751, 512), (8, 16384, 25, 16384, 2048),
         (8, 8192, 25, 8192, 2048), (4, 16384, 25, 16384, 2048), (8, 64, 24, 3, 256), (5, 4097, 25, 2600, 1024)]


@pytest.mark.parametrize("world,k,n_mod,n,chunk", CASES)
def test_strip_layout_writes_stay_in_their_regions(world, k, n_mod, n, chunk):
    ld = _res_ld(k)
    plan = plan_column_chunks(n, chunk)
    L = StripLayout(world, k, n_mod, ld, plan)
    assert L.pitch >= 2 and L.res_bytes % 256 == 0 and L.chunk_bytes % 256 == 0 and L.slot_bytes % 256 == 0
    for j, (c0, c1) in enumerate(plan):
        w = c1 - c0
        assert sum(s1 - s0 for s0, s1 in L.strips[j]) == w
        lo_chunk, hi_chunk = j * L.chunk_bytes, (j + 1) * L.chunk_bytes
        res_spans = []
        for q in range(world):
            span = L.residue_span(j, q)
            st = L.staging_span(j, q)
            if span is None:
                assert st is None
                continue
            (r0, r1), (e0, e1) = span
            assert lo_chunk <= r0 <= r1 < lo_chunk + L.res_bytes          # residues in the chunk's residue part
            assert lo_chunk + L.res_bytes <= e0 <= e1 < hi_chunk           # exponents after them
            assert r0 % 16 == 0 and e0 % 4 == 0                           # 16-byte residue rows, int32 exponents
            s0, s1 = L.strips[j][q]
            # Each plane's rows of this strip: disjoint from the other strips' rows of that plane.
            res_spans.append((s0, s1))
            a0, a1 = st
            slot0 = L.stage_off + j * L.slot_bytes
            assert slot0 <= a0 <= a1 < slot0 + L.slot_bytes
        for (a0, a1), (b0, b1) in itertools.combinations(res_spans, 2):
            assert a1 <= b0 or b1 <= a0
    assert L.stage_off == len(plan) * L.chunk_bytes and L.total == L.stage_off + len(plan) * L.slot_bytes


@pytest.mark.parametrize("world,k,n_mod,n,chunk", [(2, 70, 24, 600, 256), (3, 129, 24, 751, 512), (8, 33, 25, 300, 256)])
def test_strip_views_read_back_what_the_copies_wrote(world, k, n_mod, n, chunk):
    """Emulate the root's 2-D staging copy (k rows of the strip's width, row pitch
    `pitch` doubles) on a CPU buffer and read it back through staging_strip; write
    each strip's residues and exponents through chunk_views and check that every
    chunk is tiled exactly by its strips."""
    import torch

    ld = _res_ld(k)
    plan = plan_column_chunks(n, chunk)
    L = StripLayout(world, k, n_mod, ld, plan)
    buf = torch.zeros(L.total, dtype=torch.int8)
    B = torch.randn(k, n, dtype=torch.float64)
    for j, (c0, c1) in enumerate(plan):
        res, exps = L.chunk_views(buf, j)
        assert res.shape == (n_mod, c1 - c0, ld) and exps.shape == (c1 - c0,)
        for q, (s0, s1) in enumerate(L.strips[j]):
            off = L.stage_off + j * L.slot_bytes
            slot = buf[off: off + 8 * k * L.pitch].view(torch.float64).view(k, L.pitch)
            slot[:, : s1 - s0] = B[:, c0 + s0: c0 + s1]          # the 2-D copy
            X = L.staging_strip(buf, j, q)
            assert X.shape == (s1 - s0, k) and (s1 == s0 or X.stride() == (1, L.pitch))
            assert torch.equal(X, B[:, c0 + s0: c0 + s1].T)
            res[:, s0:s1, :] = q + 1                             # the strip's split output
            exps[s0:s1] = 1000 + q
        owner = torch.tensor([q + 1 for q, (s0, s1) in enumerate(L.strips[j]) for _ in range(s1 - s0)],
                             dtype=torch.int8)
        assert torch.equal(res[0, :, 0], owner) and torch.equal(res[-1, :, -1], owner)
        assert torch.equal(exps, owner.to(torch.int32) + 999)


@pytest.mark.parametrize("world,k,n_mod,block,strip", [(2, 700, 24, 250, 80), (8, 16384, 25, 2048, 256),
                                                       (3, 129, 24, 17, 16), (4, 64, 24, 1, 256)])
def test_column_block_layout_covers_every_column_once(world, k, n_mod, block, strip):
    """The all-gather layout: chunk c holds strip q = GPU q's columns
    [block_off[c], block_off[c] + w_c) of its block; the segmented epilogue sends
    chunk column j to C column block_off[c] + (j // w_c) * block + j % w_c.  Every
    column of C is written exactly once, by the chunk holding that GPU's piece."""
    L = StripLayout.for_blocks(world, k, n_mod, _res_ld(k), block, strip)
    assert L.slot_bytes == 0 and L.total == len(L.plan) * L.chunk_bytes
    hit = [0] * (world * block)
    for c, (c0, c1) in enumerate(L.plan):
        w = L.strips[c][0][1]
        assert c1 - c0 == world * w and L.strips[c] == [(q * w, (q + 1) * w) for q in range(world)]
        for j in range(c1 - c0):
            col = L.block_off[c] + (j // w) * block + j % w
            q = j // w
            assert q * block <= col < (q + 1) * block  # GPU q's block
            hit[col] += 1
    assert hit == [1] * (world * block)
