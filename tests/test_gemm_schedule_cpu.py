"""The tensor-core GEMM's work distribution, checked without a GPU through
the schedule functions its kernels run (lmpb_gemm_sched_tile / _unit /
_splits, exported by liblmpb.so from rushlite_b200/csrc/gemm_sm100.cu):
every output tile is produced exactly once, every k-block of a tile by
exactly one unit, the persistent CTA pairs together visit every unit, and a
forced split count never leaves a unit without k-blocks."""
from __future__ import annotations

import ctypes as C
import itertools

import pytest

from rushlite_b200 import capi


def tile(t, tiles_m, tiles_n, tm, tn):
    m0, n0 = C.c_int(), C.c_int()
    capi.lib().lmpb_gemm_sched_tile(t, tiles_m, tiles_n, tm, tn, C.byref(m0), C.byref(n0))
    return m0.value, n0.value


def units(num_tiles, splits, num_kb):
    t, kb0, kb1 = C.c_int(), C.c_int(), C.c_int()
    for u in range(num_tiles * splits):
        capi.lib().lmpb_gemm_sched_unit(u, splits, num_kb, C.byref(t), C.byref(kb0), C.byref(kb1))
        yield u, t.value, kb0.value, kb1.value


def splits_for(ntiles, num_kb, clusters, forced=0):
    return capi.lib().lmpb_gemm_sched_splits(ntiles, num_kb, clusters, forced)


@pytest.mark.parametrize("m,n", [(256, 256), (300, 260), (4096, 4096), (8192, 1000), (2048, 4096), (256, 8192),
                                 (33 * 256, 5 * 256 + 1)])
@pytest.mark.parametrize("tm", [128, 256])
def test_grouped_tile_order_is_a_bijection(m, n, tm):
    tn = 256
    tiles_m, tiles_n = -(-m // tm), -(-n // tn)
    seen = set()
    for t in range(tiles_m * tiles_n):
        m0, n0 = tile(t, tiles_m, tiles_n, tm, tn)
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
    assert sorted(per_tile) == list(range(num_tiles))
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
            m0, n0 = tile(t, tiles_m, tiles_n, 256, 256)
            for r in (0, 1):
                assert m0 <= m0 + 128 * r < m0 + 256 and n0 <= n0 + 128 * r < n0 + 256


@pytest.mark.parametrize("num_kb", range(1, 70))
@pytest.mark.parametrize("forced", [2, 3, 4, 5, 8])
def test_forced_split_count_never_leaves_a_unit_without_k_blocks(num_kb, forced):
    sp = splits_for(64, num_kb, 74, forced)
    assert 1 <= sp <= forced
    for _, _, kb0, kb1 in units(1, sp, num_kb):
        assert kb0 < kb1


def test_split_heuristic():
    # short K is never split; long K is split in two when it shortens the run
    assert splits_for(256, 128, 74) == 1          # 4096^3: 128 k-blocks
    assert splits_for(256, 256, 74) == 2          # 4096 x 8192 x 4096: 3.46 -> 6.92 rounds / 2
    assert splits_for(512, 256, 74) == 1          # 7 rounds either way: no gain
    assert splits_for(64, 1024, 74) == 1          # 64 tiles fit one round of 74 pairs either way
    assert splits_for(256, 1024, 74) == 2         # 4096 x 32768 x 4096
    assert splits_for(64, 1024, 0) == 1           # no CTA pair fits: the single-CTA kernel, unsplit
