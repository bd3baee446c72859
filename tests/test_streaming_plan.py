"""Host logic of the expert-granular streamer (no GPU): how hit experts are
cut into staged id ranges and copy runs."""

import pytest

from blockstreamer_b200.streaming import plan_groups


def test_plan_covers_every_hit_expert_once_in_order():
    hit = [0, 1, 2, 5, 6, 9, 10, 11, 12, 20]
    plan = plan_groups(hit, 3)
    assert len(plan) == 3
    seen = [e for _, _, runs in plan for a, b in runs for e in range(a, b)]
    assert seen == hit
    for e0, e1, runs in plan:
        assert e0 == runs[0][0] and e1 == runs[-1][1]
    # ranges are disjoint and ascending
    assert all(plan[i][1] <= plan[i + 1][0] for i in range(len(plan) - 1))


def test_plan_merges_consecutive_ids_into_runs():
    plan = plan_groups([3, 4, 5, 7, 8], 1)
    assert plan == [(3, 9, [(3, 6), (7, 9)])]


def test_plan_balances_expert_counts():
    plan = plan_groups(list(range(0, 128, 1)), 4)
    sizes = [sum(b - a for a, b in runs) for _, _, runs in plan]
    assert sizes == [32, 32, 32, 32]
    plan = plan_groups(list(range(10)), 4)
    sizes = [sum(b - a for a, b in runs) for _, _, runs in plan]
    assert sorted(sizes) == [2, 2, 3, 3] and sum(sizes) == 10


def test_plan_edge_cases():
    assert plan_groups([], 4) == []
    assert plan_groups([7], 4) == [(7, 8, [(7, 8)])]          # fewer experts than groups
    assert plan_groups([2, 2, 1], 2) == [(1, 2, [(1, 2)]), (2, 3, [(2, 3)])]   # duplicates, unsorted
    with pytest.raises(ValueError):
        plan_groups([1], 0)
