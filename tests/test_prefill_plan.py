"""The prefill schedule (``hyt_prefill_plan``), a host function: no GPU needed.

Every work item of the default grid (request, query tile, head pair) must appear exactly
once, whole, or as two halves that cover its key tiles [0, n) with one split slot; the
order is longest first; the default grid is kept when nothing beats it.
"""

from __future__ import annotations

import math
import random

import numpy as np
import pytest

from hayate_b200 import ops


def key_tiles(cache_len, q_len, qt):
    t_last = min(qt * 128 + 127, q_len - 1)
    return (cache_len + t_last) // 128 + 1


def check_cover(items, splits, cache_lens, q_lens, heads):
    seen = {}
    for z, tp, keys, split in items.tolist():
        qt, pair = tp & 0xFFFF, tp >> 16
        lo, hi = keys & 0xFFFF, keys >> 16
        seen.setdefault((z, qt, pair), []).append((lo, hi, split))
    expect = {(z, qt, pair) for z, ql in enumerate(q_lens) for qt in range(math.ceil(ql / 128))
              for pair in range(heads // 2)}
    assert set(seen) == expect
    slots = set()
    for (z, qt, pair), parts in seen.items():
        n = key_tiles(cache_lens[z], q_lens[z], qt)
        if len(parts) == 1:
            assert parts[0] == (0, n, -1)
        else:
            (lo0, hi0, s0), (lo1, hi1, s1) = sorted(parts)
            assert lo0 == 0 and hi0 == lo1 and hi1 == n and s0 >> 1 == s1 >> 1
            assert {s0 & 1, s1 & 1} == {0, 1}
            slots.add(s0 >> 1)
    assert slots == set(range(splits))


@pytest.mark.parametrize("seed", range(6))
def test_plan_covers_every_item_once(seed):
    rng = random.Random(seed)
    cache_lens = [rng.randint(0, 8192) for _ in range(rng.randint(1, 12))]
    q_lens = [512] * len(cache_lens)
    items, splits = ops.prefill_plan(cache_lens, 512, 32, 148, 128)
    if items is None:
        assert splits == 0
        return
    check_cover(items, splits, cache_lens, q_lens, 32)
    assert splits <= 128
    # longest first: the halves (which also pay the merge, 8 key tiles in the cost model)
    # and whole items in non-increasing cost order
    costs = [((k >> 16) - (k & 0xFFFF)) + (8.0 if s >= 0 else 0.0) for _, _, k, s in items.tolist()]
    assert all(a >= b - 1e-9 for a, b in zip(costs, costs[1:]))


def test_plan_packed_lengths_and_limits():
    cache_lens = [0, 5000, 300, 12000]
    q_lens = [700, 130, 1, 512]
    items, splits = ops.prefill_plan(cache_lens, 0, 32, 148, 16, q_lens=q_lens)
    assert items is not None
    check_cover(items, splits, cache_lens, q_lens, 32)
    assert splits <= 16
    none, zero = ops.prefill_plan(cache_lens, 0, 32, 148, 0, q_lens=q_lens)  # no splits allowed
    if none is not None:
        check_cover(none, zero, cache_lens, q_lens, 32)
        assert zero == 0


def test_plan_keeps_default_grid_when_it_is_as_good():
    # one item per SM or fewer, all the same size: nothing to gain from reordering; a
    # split would double the CTAs, so with no splits allowed the default grid stays
    items, splits = ops.prefill_plan([1024] * 4, 128, 32, 148, 0)
    assert items is None and splits == 0


def test_plan_rejects_bad_arguments():
    with pytest.raises(RuntimeError):
        ops.prefill_plan([10, 20], 0, 32, 148, 8)  # no q_lens and query_len 0
    assert ops.prefill_workspace_bytes(0) == 0
    assert ops.prefill_workspace_bytes(3) >= 3 * 266240


def model_choice(cache_lens, q_len, pairs, sms, max_splits, ov=5.0, mc=8.0, min_gain=0.03):
    """The planner's decision restated: greedy makespans of the default grid and of
    longest-first orders with the k heaviest items cut; returns the chosen k or None."""
    import heapq

    def makespan(costs):
        free = [0.0] * sms
        end = 0.0
        for c in costs:
            t = heapq.heappop(free) + c
            heapq.heappush(free, t)
            end = max(end, t)
        return end

    base = []
    for z, cl in enumerate(cache_lens):
        tiles = -(-q_len // 128)
        for pair in range(pairs):
            for qt in reversed(range(tiles)):
                base.append(key_tiles(cl, q_len, qt))
    grid = makespan([n + ov for n in base])
    lpt = sorted(base, key=lambda n: -(n + ov))  # stable, like the C++ stable_sort
    splittable = sum(n >= 2 for n in lpt)
    best, best_k = grid, None
    for k in (0, 8, 16, 24, 32, 48, 64, 96, 128, 192, 256, 384, 512):
        if k > min(max_splits, splittable):
            break
        costs, slot = [], 0
        for n in lpt:
            if slot < k and n >= 2:
                costs += [n // 2 + ov + mc, (n - n // 2) + ov + mc]
                slot += 1
            else:
                costs.append(n + ov)
        m = makespan(sorted(costs, reverse=True))
        if m < best - 1e-9:
            best, best_k = m, k
    if best_k is None or best > (1 - min_gain) * grid:
        return None
    return best_k


@pytest.mark.parametrize("seed", range(8))
def test_plan_choice_matches_the_model(seed):
    rng = random.Random(100 + seed)
    cache_lens = [rng.randint(0, rng.choice([4096, 16384, 32768])) for _ in range(rng.randint(1, 8))]
    expect = model_choice(cache_lens, 512, 16, 148, 128)
    items, splits = ops.prefill_plan(cache_lens, 512, 32, 148, 128)
    if expect is None:
        assert items is None
    else:
        assert items is not None and splits == expect
