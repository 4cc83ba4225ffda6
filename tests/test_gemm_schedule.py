"""CPU: the integer invariants the GEMM kernel's stream-K schedule relies on, checked on the
kernel's own code.

The persistent W8A16 kernel (csrc/gemm.cu: ``sk_start``, ``sk_owner``, ``SegWalk``, ``sk_pieces``,
all ``__host__ __device__``) lays every output tile's k-blocks end to end (tile-major) and gives
CTA b the range [b * W / G, (b + 1) * W / G).  A tile cut by a range boundary is finished by the
CTAs that share it: each writes its piece to slot [cta][0] (its first segment) or [cta][1] (a later
one), counts on the counter of the CTA holding the tile's first k-block, and the last arriver sums
the pieces in k order.  The library's host-only ``bw_debug_streamk_*`` entry points run that same
code; over many (k-blocks, tiles, grid) shapes this checks: every k-block is covered once; a cut
tile's contributors are consecutive CTAs from its first k-block's owner on, in k order, and their
count and first slot are what ``sk_pieces`` (the kernel's epilogue) says; no two pieces share a
slot; each CTA heads at most one cut tile (so per-CTA counters suffice); only the first contributor
can hold a cut tile as a later segment (slot 1); the owner of every k-block is the CTA whose range
holds it.
"""
import ctypes
import itertools

import pytest

SHAPES = [(kb, tiles, g) for kb, tiles, g in itertools.product([1, 2, 3, 7, 8, 24, 64, 224], [1, 3, 8, 24, 224, 1187],
                                                                [148, 96, 7])
          if kb * tiles >= g]


@pytest.fixture(scope="module")
def lib():
    from blackwell_ops import _lib

    return _lib.lib


def _walk(lib, kb, tiles, g, b):
    room = tiles + 2  # a CTA's range touches at most every tile once
    buf = (ctypes.c_int32 * (4 * room))()
    n = lib.bw_debug_streamk_walk(kb, tiles, g, b, ctypes.cast(buf, ctypes.c_void_p), room)
    assert n >= 0
    return [tuple(buf[4 * i:4 * i + 4]) for i in range(n)]


@pytest.mark.parametrize("kb,tiles,g", SHAPES)
def test_stream_k_schedule_invariants(lib, kb, tiles, g):
    w = kb * tiles
    assert w * g < 2 ** 31  # the kernel's 32-bit range arithmetic
    start = [lib.bw_debug_streamk_start(kb, tiles, g, b) for b in range(g + 1)]
    assert start[0] == 0 and start[g] == w
    cover = [0] * w
    pieces, slots = {}, set()
    for b in range(g):
        assert start[b] < start[b + 1]  # no empty range when the grid is at most the work
        for t, k0, nkb, split in _walk(lib, kb, tiles, g, b):
            for k in range(k0, k0 + nkb):
                cover[t * kb + k] += 1
            if nkb < kb:
                pieces.setdefault(t, []).append((b, k0, split))
                assert (b, split) not in slots
                slots.add((b, split))
    assert all(c == 1 for c in cover)
    heads = set()
    loc = (ctypes.c_int32 * 3)()
    for t, ps in pieces.items():
        assert lib.bw_debug_streamk_pieces(kb, tiles, g, t, ctypes.cast(loc, ctypes.c_void_p)) == 0
        b0, n_parts, slot0 = loc[0], loc[1], loc[2]
        assert [p[0] for p in ps] == list(range(b0, b0 + n_parts))
        assert [p[1] for p in ps] == sorted(p[1] for p in ps)
        assert ps[0][2] == slot0
        for b, _, split in ps:
            assert split == (0 if start[b] // kb == t else 1)
            if b != b0:
                assert split == 0
        assert b0 not in heads
        heads.add(b0)
    for x in range(0, w, max(1, w // 499)):
        o = lib.bw_debug_streamk_owner(kb, tiles, g, x)
        assert start[o] <= x < start[o + 1]


def test_debug_entry_points_reject_bad_plans(lib):
    buf = (ctypes.c_int32 * 8)()
    p = ctypes.cast(buf, ctypes.c_void_p)
    assert lib.bw_debug_streamk_walk(1, 1, 2, 0, p, 2) == -1      # less work than CTAs
    assert lib.bw_debug_streamk_walk(8, 8, 4, 4, p, 2) == -1      # no such CTA
    assert lib.bw_debug_streamk_walk(64, 1187, 148, 0, p, 1) == -1  # more segments than room
    assert lib.bw_debug_streamk_owner(8, 8, 4, 64) == -1
