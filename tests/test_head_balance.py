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


@pytest.mark.parametrize("world", [2, 3, 4, 5, 8, 16])
def test_free_size_partition_is_valid_and_deterministic(world):
    rnd = random.Random(100 + world)
    scores = [rnd.lognormvariate(0, 1) for _ in range(16)]
    groups = shard.balanced_heads(scores, world, cap=2.0, equal_size=False)
    assert len(groups) == world and all(len(g) >= 1 and g == sorted(g) for g in groups)
    assert sorted(h for g in groups for h in g) == list(range(16))
    assert groups == shard.balanced_heads(list(scores), world, cap=2.0, equal_size=False)


def _cost_max(shares, groups, head_cost):
    return max(sum(shares[h] + head_cost for h in g) for g in groups)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_free_size_partition_is_no_worse_than_equal_size(world):
    """Under the work model it balances (a fixed cost per head plus its
    expected budget), free sizes never lose to equal sizes and stay close to
    the lower bound max(heaviest head, mean load)."""
    for seed in range(30):
        rnd = random.Random(seed)
        scores = [rnd.lognormvariate(0, 1) for _ in range(16)]
        s = shard.budget_shares(scores, 2.0)
        free = shard.balanced_heads(scores, world, 2.0, equal_size=False)
        equal = shard.balanced_heads(scores, world, 2.0)
        c = shard.HEAD_COST
        got, eq = _cost_max(s, free, c), _cost_max(s, equal, c)
        bound = max(max(x + c for x in s), sum(x + c for x in s) / world)
        assert got <= eq + 1e-9
        assert got <= 1.34 * bound, (seed, got, bound)


def test_free_size_partition_of_the_bench_layer():
    """The cfg2 bench layer's head scores over 8 ranks: the two capped heads
    sit on different ranks, and the worst rank is within 13 % of the mean
    (a capped head plus the fixed cost of a second head is already 1.12 x the
    mean) and no worse than the equal-size partition."""
    import torch
    from ress_b200 import synth

    cam, pcd = synth.fisher_table(seed=1)[0], synth.fisher_table(seed=3)[0]
    comb = 0.5 * cam / cam.sum(-1, keepdim=True) + 0.5 * pcd / pcd.sum(-1, keepdim=True)
    hs = (comb / comb.sum(-1, keepdim=True))[0].tolist()
    groups = shard.balanced_heads(hs, 8, cap=2.0, equal_size=False)
    s = shard.budget_shares(hs, 2.0)
    c = shard.HEAD_COST
    assert not any(0 in g and 9 in g for g in groups)
    mean = sum(x + c for x in s) / 8
    assert _cost_max(s, groups, c) <= 1.13 * mean
    assert _cost_max(s, groups, c) <= _cost_max(s, shard.balanced_heads(hs, 8, cap=2.0), c) + 1e-9
