"""CPU: the integer invariants the GEMM kernel's stream-K schedule relies on.

The persistent W8A16 kernel (csrc/gemm.cu, ``sk_start`` / ``sk_owner`` / ``SegWalk``)
lays every output tile's k-blocks end to end (tile-major) and gives CTA b the
range [b * W / G, (b + 1) * W / G).  A tile cut by a range boundary is finished by
the CTAs that share it: each writes its piece to slot [cta][0] (its first
segment) or [cta][1] (a later one), counts on the counter of the CTA holding the
tile's first k-block, and the last arriver sums the pieces in k order.  This
restates that arithmetic and checks, over many (k-blocks, tiles, grid) shapes:
every k-block is covered once; a cut tile's contributors are consecutive CTAs
from its first k-block's owner on, in k order; no two pieces share a slot; each
CTA heads at most one cut tile (so per-CTA counters suffice); and only the first
contributor can hold a cut tile as a later segment (slot 1).
"""
import itertools

import pytest


def start(b, w, g):
    return b * w // g


def owner(x, w, g):
    return ((x + 1) * g + w - 1) // w - 1


def walk(b, w, g, kb):
    x, end, first = start(b, w, g), start(b + 1, w, g), True
    while x < end:
        t = x // kb
        t0 = t * kb
        k0 = x - t0
        nkb = min(kb, end - t0) - k0
        yield t, k0, nkb, 0 if first else 1
        first = False
        x = t0 + k0 + nkb


SHAPES = [(kb, tiles, g) for kb, tiles, g in itertools.product([1, 2, 3, 7, 8, 24, 64, 224], [1, 3, 8, 24, 224, 1187],
                                                                [148, 96, 7])
          if kb * tiles >= g]


@pytest.mark.parametrize("kb,tiles,g", SHAPES)
def test_stream_k_schedule_invariants(kb, tiles, g):
    w = kb * tiles
    assert w * g < 2 ** 31  # the kernel's 32-bit range arithmetic
    cover = [0] * w
    pieces, slots = {}, set()
    for b in range(g):
        assert start(b, w, g) < start(b + 1, w, g)  # no empty range when the grid is at most the work
        for t, k0, nkb, split in walk(b, w, g, kb):
            for k in range(k0, k0 + nkb):
                cover[t * kb + k] += 1
            if nkb < kb:
                pieces.setdefault(t, []).append((b, k0, split))
                assert (b, split) not in slots
                slots.add((b, split))
    assert all(c == 1 for c in cover)
    heads = set()
    for t, ps in pieces.items():
        b0, b1 = owner(t * kb, w, g), owner(t * kb + kb - 1, w, g)
        assert [p[0] for p in ps] == list(range(b0, b1 + 1))
        assert [p[1] for p in ps] == sorted(p[1] for p in ps)
        for b, _, split in ps:
            assert split == (0 if start(b, w, g) // kb == t else 1)
            if b != b0:
                assert split == 0
        assert b0 not in heads
        heads.add(b0)
    for x in range(0, w, max(1, w // 499)):
        o = owner(x, w, g)
        assert start(o, w, g) <= x < start(o + 1, w, g)
