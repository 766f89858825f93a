"""Host model of the tensor-core GEMM's work distribution (the index
arithmetic of tile_coords / tile_coords_pair and the split-K unit ranges in
rushlite_b200/csrc/gemm_sm100.cu), checked without a GPU: every output tile
is produced exactly once, every k-block of a tile by exactly one unit, and
the persistent CTAs (pairs) together visit every unit."""
from __future__ import annotations

import itertools

import pytest


def tile_coords(t, tiles_m, tiles_n, tm, tn, group=8):
    g = t // (group * tiles_n)
    first_m = g * group
    gsize = min(tiles_m - first_m, group)
    local = t % (group * tiles_n)
    return (first_m + local % gsize) * tm, (local // gsize) * tn


def clamp_splits(splits, num_kb):
    """The host's rule for a forced split count: at most one per k-block, and
    no unit without a k-block."""
    splits = max(1, min(splits, max(1, num_kb)))
    while splits > 1 and (splits - 1) * (-(-num_kb // splits)) >= num_kb:
        splits -= 1
    return splits


def units(num_tiles, splits, num_kb):
    kb_per = (num_kb + splits - 1) // splits
    for u in range(num_tiles * splits):
        t, ks = divmod(u, splits)
        kb0 = ks * kb_per
        yield u, t, kb0, min(num_kb, kb0 + kb_per)


@pytest.mark.parametrize("m,n", [(256, 256), (300, 260), (4096, 4096), (8192, 1000), (2048, 4096), (256, 8192),
                                 (33 * 256, 5 * 256 + 1)])
@pytest.mark.parametrize("tm", [128, 256])
def test_grouped_tile_order_is_a_bijection(m, n, tm):
    tn = 256
    tiles_m, tiles_n = -(-m // tm), -(-n // tn)
    seen = set()
    for t in range(tiles_m * tiles_n):
        m0, n0 = tile_coords(t, tiles_m, tiles_n, tm, tn)
        assert 0 <= m0 < tiles_m * tm and 0 <= n0 < tiles_n * tn
        assert m0 % tm == 0 and n0 % tn == 0
        seen.add((m0, n0))
    assert len(seen) == tiles_m * tiles_n


@pytest.mark.parametrize("num_tiles,splits,num_kb,pairs", [(256, 2, 256, 74), (256, 3, 128, 74), (64, 4, 1024, 74),
                                                           (1, 2, 9, 74), (1024, 1, 256, 74), (5, 2, 33, 3)])
def test_split_units_partition_k_and_pairs_cover_units(num_tiles, splits, num_kb, pairs):
    per_tile = {}
    for u, t, kb0, kb1 in units(num_tiles, splits, num_kb):
        assert kb0 < kb1, "every unit has at least one k-block"
        per_tile.setdefault(t, []).append((kb0, kb1))
    for t, ranges in per_tile.items():
        ranges.sort()
        assert ranges[0][0] == 0 and ranges[-1][1] == num_kb
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
    grid = min(num_tiles * splits, pairs)
    visited = sorted(itertools.chain.from_iterable(range(p, num_tiles * splits, grid) for p in range(grid)))
    assert visited == list(range(num_tiles * splits))


def test_tma_row_coordinates_of_a_pair_stay_in_its_tile():
    # CTA rank r of a pair loads rows m0 + 128 r .. +127 of A and n0 + 128 r .. of B
    for tiles_m, tiles_n in [(3, 2), (16, 16), (1, 5)]:
        for t in range(tiles_m * tiles_n):
            m0, n0 = tile_coords(t, tiles_m, tiles_n, 256, 256)
            for r in (0, 1):
                assert m0 <= m0 + 128 * r < m0 + 256 and n0 <= n0 + 128 * r < n0 + 256


@pytest.mark.parametrize("num_kb", range(1, 70))
@pytest.mark.parametrize("forced", [2, 3, 4, 5, 8])
def test_forced_split_count_never_leaves_a_unit_without_k_blocks(num_kb, forced):
    sp = clamp_splits(forced, num_kb)
    assert 1 <= sp <= forced
    for _, _, kb0, kb1 in units(1, sp, num_kb):
        assert kb0 < kb1
