"""CPU: the persistent tensor-core kernels' work decomposition (tail split policy), checked through the
library's own planner and unit decoder (vk_debug_schedule, no device): every (tile, k-block) is computed
exactly once, slices are contiguous k-ranges of at least 4 k-blocks, the tail fits one wave, and the
slices-first ordering follows its stated conditions.  The reference's last-wave split
(results/ralph_loop_fable/src/matmul_f16/matmul_f16_v23_wavesplit.cu:1-8) had no such check."""
import itertools

import pytest

MIN_SLICE_KB = 4
MAX_SPLIT = 8


def _check(vk, tiles, num_kb, max_units, k, split=True, nsplit=True, first=True):
    plan, units = vk.debug_schedule(tiles, num_kb, max_units, k, split, nsplit, first)
    assert plan["units"] == len(units)
    assert plan["grid_units"] == min(plan["units"], max_units)
    by_tile = {}
    for tile, kb0, kb1, tag in units:
        assert 0 <= tile < tiles
        by_tile.setdefault(tile, []).append((kb0, kb1, tag))
    assert sorted(by_tile) == list(range(tiles)), "every tile appears"
    tail_tiles = 0
    for tile, parts in by_tile.items():
        tags = sorted(t for _, _, t in parts)
        if tags == [-1]:
            assert parts[0][:2] == (0, num_kb)
            continue
        tail_tiles += 1
        if tags == [100, 101]:  # column halves: both over the full k-range
            assert all(p[:2] == (0, num_kb) for p in parts)
            continue
        s = len(parts)
        assert tags == list(range(s)) and 2 <= s <= MAX_SPLIT, tags
        ranges = sorted((t, kb0, kb1) for kb0, kb1, t in parts)
        assert ranges[0][1] == 0 and ranges[-1][2] == num_kb
        for (_, _, end), (_, start, _) in zip(ranges, ranges[1:]):
            assert end == start, "slices are contiguous, no gap or overlap"
        assert all(kb1 - kb0 >= MIN_SLICE_KB for _, kb0, kb1 in ranges)
    # whole tiles: exactly full_units of them; tail units all fit one wave of clusters
    whole = sum(1 for *_, t in units if t == -1)
    assert whole == plan["full_units"]
    assert plan["units"] - whole <= max_units
    # cluster c runs units c, c + G, c + 2G, ... (G clusters launched): work per cluster, in k-blocks of a
    # whole-width tile (a column half counts half), differs by at most one tile's worth
    g = plan["grid_units"]
    work = [0.0] * g
    for u, (_, kb0, kb1, tag) in enumerate(units):
        work[u % g] += (kb1 - kb0) * (0.5 if tag >= 100 else 1.0)
    assert max(work) - min(work) <= num_kb
    if plan["tail_first"]:
        assert k >= 2560 and 2 <= plan["split"] <= 4 and plan["full_units"] >= max_units
        n_tail = plan["units"] - plan["full_units"]
        assert all(t != -1 for *_, t in units[:n_tail]), "slices are numbered before whole tiles"
        assert all(t == -1 for *_, t in units[n_tail:])
    else:
        assert all(t == -1 for *_, t in units[:plan["full_units"]]), "whole tiles come first"
    return plan


@pytest.mark.parametrize("max_units", [74, 148, 37, 1])
def test_schedule_covers_every_tile_and_k_block_once(max_units):
    import vibekernel_b200 as vk
    for tiles, num_kb in itertools.product([1, 2, 16, 33, 64, 73, 74, 75, 100, 148, 256, 300, 1024],
                                           [1, 3, 4, 7, 8, 16, 24, 32, 64]):
        for k in (num_kb * 128, 1000):
            for flags in ((True, True, True), (True, False, True), (True, True, False), (False, True, True)):
                _check(vk, tiles, num_kb, max_units, k, *flags)


def test_schedule_policies_on_the_bench_shapes():
    import vibekernel_b200 as vk
    # 4096^3 on 74 pair clusters: 3 whole waves + 34 tiles in 2 slices, run first
    plan = _check(vk, 256, 32, 74, 4096)
    assert (plan["full_units"], plan["split"], plan["tail_first"]) == (222, 2, 1)
    # 4000x5120x3000: 16 x 20 tiles, 24 k-blocks: 4 waves + 24 tiles in 3 slices, run first
    plan = _check(vk, 320, 24, 74, 3000)
    assert (plan["full_units"], plan["split"], plan["tail_first"]) == (296, 3, 1)
    # K = 1024 (8 k-blocks): too shallow to run slices first -> column halves of the 34 tail tiles
    plan = _check(vk, 256, 8, 74, 1024)
    assert (plan["nsplit"], plan["tail_first"], plan["units"]) == (1, 0, 222 + 68)
    # 1024^3: 16 tiles on 74 clusters, no whole wave, 8 k-blocks: only 2 slices would fit -> column halves
    plan = _check(vk, 16, 8, 74, 1024)
    assert (plan["nsplit"], plan["split"], plan["full_units"], plan["units"]) == (1, 1, 0, 32)
    # 1024 x 1024 x 8192: 16 tiles, 64 k-blocks: 4 k-slices per tile (R <= C/4), no whole wave to run before
    plan = _check(vk, 16, 64, 74, 8192)
    assert (plan["split"], plan["tail_first"], plan["units"]) == (4, 0, 64)
    # 8192^3: 1024 tiles, 62 left over: neither halves (2R > C) nor slices (C / R = 1)
    plan = _check(vk, 1024, 64, 74, 8192)
    assert (plan["split"], plan["nsplit"], plan["units"]) == (1, 0, 1024)
    # tail split switched off: whole tiles only
    plan = _check(vk, 256, 32, 74, 4096, split=False)
    assert plan["units"] == 256 and plan["split"] == 1 and plan["nsplit"] == 0


def test_schedule_hook_rejects_bad_arguments():
    import vibekernel_b200 as vk
    with pytest.raises(vk.VkError):
        vk.debug_schedule(10, 0, 74, 4096)
    with pytest.raises(vk.VkError):
        vk.debug_schedule(10, 4, 0, 4096)
