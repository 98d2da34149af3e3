"""Host-side tiling of a prefill batch for cdb_prefill_attention (OuroRunner.prefill_tiles).

A tile is a run of at most 64 consecutive positions of one request: {row_start, rows, slot,
position of row_start}. Tiles come longest-attention-first (keys attended = position + rows), so
the kernel's CTAs, which start in tile order, begin with the heaviest work. Every prompt row is in
exactly one tile whatever the order.
"""

from __future__ import annotations

import random

from continuous_depth_batching_b200.runner import OuroRunner


def _batch(seed: int):
    rng = random.Random(seed)
    slots, pos = [], []
    for slot in rng.sample(range(64), 12):
        start = rng.choice([0, 0, 17, 40])  # fresh prompts and chunks after cached tokens
        n = rng.randint(1, 300)
        slots += [slot] * n
        pos += list(range(start, start + n))
    return slots, pos


def test_tiles_cover_every_row_once_in_runs_of_one_request():
    for seed in range(5):
        slots, pos = _batch(seed)
        tiles = OuroRunner.prefill_tiles(slots, pos)
        seen = []
        for row0, n, slot, p0 in tiles:
            assert 1 <= n <= 64
            for i in range(n):
                assert slots[row0 + i] == slot and pos[row0 + i] == p0 + i
            seen += range(row0, row0 + n)
        assert sorted(seen) == list(range(len(slots)))


def test_tiles_ordered_by_attended_keys():
    slots, pos = _batch(7)
    tiles = OuroRunner.prefill_tiles(slots, pos)
    keys = [p0 + n for _row0, n, _slot, p0 in tiles]
    assert keys == sorted(keys, reverse=True)
    # ties keep row order (stable)
    for a, b in zip(tiles, tiles[1:]):
        if a[3] + a[1] == b[3] + b[1]:
            assert a[0] < b[0]
