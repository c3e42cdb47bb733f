"""Placement of hot experts over the GPUs of a node (host logic)."""
import numpy as np

from xtier_b200.cache.peer import owners, plan_sets


def test_plan_sets_cover_and_replicate():
    E, budget = 128, 51
    pop = np.random.default_rng(0).random(E)
    order = list(np.argsort(-pop))
    for W in (1, 2, 4, 8):
        sets = plan_sets(E, budget, W, pop)
        assert len(sets) == W and all(len(s) == budget for s in sets)
        assert all(len(set(s)) == budget for s in sets)
        common = set.intersection(*map(set, sets))
        assert set(order[:budget // 2]) <= common          # the most popular are on every GPU
        union = set().union(*map(set, sets))
        if budget * W >= E and W > 1:
            assert union == set(range(E)), W                # the node's slots cover every expert
    assert plan_sets(E, budget, 1, pop)[0] == order[:budget]


def test_owners_prefer_local_copy():
    sets = [[5, 1, 2], [5, 3, 4]]
    own = owners(sets, 1)
    assert own[5] == (1, 0) and own[3] == (1, 1) and own[1] == (0, 1) and own[2] == (0, 2)
    assert 7 not in own
