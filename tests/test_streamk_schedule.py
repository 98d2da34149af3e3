"""Stream-K schedule invariants of the tcgen05 GEMM (csrc/gemm.cu, csrc/gemm_pair.cuh), on the CPU.

The kernels cut the (tile, 64-wide k block) iteration space into G equal contiguous ranges (G CTAs
in the one-SM mode, G CTA pairs in the pair mode) with `range_start`, find the range holding an
iteration with `cta_of`, and place split-tile pieces in workspace slots with `piece_slot`. A tile
split over ranges is finished by its owner (the range holding its first k block), which waits
until `gb - ga` pieces have been counted on the tile's counter and then reads the pieces of ranges
ga+1 .. gb from slots 2(ga+1), 2(ga+2), ... This restates those three formulas and the segment walk
of `PairWork` and checks what the fixup relies on, for the launch sizes the host allows (at most
`iters` ranges; the pair mode also needs two tiles per pair): every (tile, k block) is done once,
the owner's segment is the last of its range, every other piece is the first segment of its range
and lands in slot 2g, and the number of pieces published equals the number the owner waits for.
An empty range breaks the last point (an owner would count it and wait for a piece that never
comes), which is why the host never launches more ranges than iterations.
"""

from __future__ import annotations

import pytest


def range_start(iters: int, G: int, g: int) -> int:
    return iters * g // G


def cta_of(iters: int, G: int, x: int) -> int:
    return ((x + 1) * G - 1) // iters


def piece_slot(iters: int, G: int, g: int, tile_begin: int) -> int:
    return 2 * g if range_start(iters, G, g) >= tile_begin else 2 * g + 1


def segments(tiles: int, kb: int, G: int, g: int):
    """(tile, first k, end k) runs of range g, in order (PairWork::at / seg_end)."""

    iters = tiles * kb
    it0, it1 = range_start(iters, G, g), range_start(iters, G, g + 1)
    it = it0
    while it < it1:
        t = it // kb
        e = min((t + 1) * kb, it1)
        yield t, it - t * kb, e - t * kb
        it = e


def check_schedule(tiles: int, kb: int, G: int) -> int:
    iters = tiles * kb
    done = {}
    owners, pieces = {}, {}
    for g in range(G):
        segs = list(segments(tiles, kb, G, g))
        assert segs, f"range {g} is empty"
        for n, (t, k0, k1) in enumerate(segs):
            for k in range(k0, k1):
                done[(t, k)] = done.get((t, k), 0) + 1
            if k0 == 0 and k1 == kb:
                continue  # whole tile, stored directly
            tb = t * kb
            ga, gb = cta_of(iters, G, tb), cta_of(iters, G, tb + kb - 1)
            assert ga <= g <= gb
            if g == ga:
                assert n == len(segs) - 1, "the owner's piece is its range's last segment"
                owners[t] = gb - ga
                first = piece_slot(iters, G, ga + 1, tb)
                assert [first + 2 * i for i in range(gb - ga)] == [2 * h for h in range(ga + 1, gb + 1)]
            else:
                assert n == 0, "a non-owner piece is its range's first segment"
                slot = piece_slot(iters, G, g, tb)
                assert slot == 2 * g and slot < 2 * G
                pieces.setdefault(t, []).append(g)
    assert all(done.get((t, k)) == 1 for t in range(tiles) for k in range(kb))
    assert all(len(pieces.get(t, [])) == n for t, n in owners.items())
    return len(owners)


@pytest.mark.parametrize("kb", [1, 2, 3, 8, 9, 32, 88])
def test_one_sm_mode_schedules(kb):
    # one CTA per SM, capped at the iteration count (shape_for)
    for tiles in list(range(1, 120)) + [256, 768, 1408]:
        for sms in (148, 147, 74, 7, 1):
            check_schedule(tiles, kb, min(sms, tiles * kb))


@pytest.mark.parametrize("kb", [1, 2, 3, 8, 32, 88])
def test_pair_mode_schedules(kb):
    # pairs = min(SMs / 2, resident clusters, iterations), taken only with two tiles per pair
    for tiles in list(range(2, 260)) + [768, 1408]:
        for pairs in (74, 73, 70, 37, 2, 1):
            G = min(pairs, tiles * kb)
            if tiles >= 2 * G:
                check_schedule(tiles, kb, G)


def test_bench_prefill_shapes_split_tiles():
    # the 8192-token projections of Ouro-1.4B on 74 pairs: QKV, o_proj, gate/up, down
    for n, k in ((6144, 2048), (2048, 2048), (11264, 2048), (2048, 5632)):
        tiles = (n // 256) * (8192 // 256)
        split = check_schedule(tiles, k // 64, 74)
        assert 0 < split < 74  # at most one split tile per range boundary


def test_more_ranges_than_iterations_leave_a_range_empty():
    # the launch sizes the host avoids: with 7 ranges over 4 iterations some ranges are empty
    with pytest.raises(AssertionError, match="empty"):
        check_schedule(2, 2, 7)
