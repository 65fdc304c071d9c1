"""The head partition of the multi-GPU head split (shard.balanced_heads over
shard.budget_shares): host logic, no GPU.  Every rank must compute the same
partition into equal-size groups, and the greedy pass must stay close to the
best partition (checked by brute force on 8 heads)."""

import itertools
import random

import pytest

from ress_b200 import shard


def _partitions(items, size):
    if not items:
        yield []
        return
    first = items[0]
    for rest in itertools.combinations(items[1:], size - 1):
        left = [x for x in items[1:] if x not in rest]
        for p in _partitions(left, size):
            yield [(first, *rest)] + p


def _max_load(shares, groups):
    return max(sum(shares[h] for h in g) for g in groups)


@pytest.mark.parametrize("world", [1, 2, 4, 8, 16])
def test_partition_is_valid_and_deterministic(world):
    rnd = random.Random(world)
    scores = [rnd.lognormvariate(0, 1) for _ in range(16)]
    groups = shard.balanced_heads(scores, world, cap=2.0)
    assert len(groups) == world
    assert all(len(g) == 16 // world and g == sorted(g) for g in groups)
    assert sorted(h for g in groups for h in g) == list(range(16))
    assert groups == shard.balanced_heads(list(scores), world, cap=2.0)


def test_uneven_split_is_rejected():
    with pytest.raises(ValueError):
        shard.balanced_heads([1.0] * 16, 3)


def test_shares_sum_to_head_count_and_respect_the_cap():
    rnd = random.Random(7)
    for _ in range(50):
        scores = [rnd.lognormvariate(0, 1.5) for _ in range(16)]
        for cap in (None, 1.5, 2.0, 4.0):
            w = shard.budget_shares(scores, cap)
            assert abs(sum(w) - 16.0) < 1e-9
            if cap is not None:
                assert max(w) <= cap + 1e-9


@pytest.mark.parametrize("world", [2, 4])
def test_greedy_is_close_to_the_best_partition(world):
    worst = 1.0
    for seed in range(40):
        rnd = random.Random(seed)
        scores = [rnd.lognormvariate(0, 1) for _ in range(8)]
        for cap in (None, 2.0):
            s = shard.budget_shares(scores, cap)
            got = _max_load(s, shard.balanced_heads(scores, world, cap))
            best = min(_max_load(s, p) for p in _partitions(list(range(8)), 8 // world))
            assert got >= best - 1e-12
            worst = max(worst, got / best)
    assert worst <= 4.0 / 3.0, worst
