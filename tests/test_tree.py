"""Draft trees on the CPU (runtime/tree.py): chains merged into one trie under the root, the node budget with
ancestors kept, breadth-first order, ancestor words, and the greedy walk."""
import numpy as np

from xtier_b200.runtime.tree import Tree, build_tree, walk_greedy


def test_merge_budget_and_order():
    t = build_tree(7, [([1, 2, 3], [1.0, 1.0, 1.0]), ([1, 5], [0.9, 0.8]), ([4, 4], [0.5, 0.5])], budget=16)
    # root, 1, 4 at depth 1; 2, 5, 4 at depth 2; 3 at depth 3: the shared prefix [1] is one node
    assert t.n == 7 and int(t.tokens[0]) == 7 and int(t.parents[0]) == -1
    assert list(t.depth) == sorted(t.depth)                          # breadth-first
    assert all(t.parents[i] < i for i in range(1, t.n))             # parents before children
    one = [i for i in range(t.n) if int(t.tokens[i]) == 1]
    assert len(one) == 1 and sorted(int(t.tokens[c]) for c in t.children(one[0])) == [2, 5]
    small = build_tree(7, [([1, 2, 3], [1.0] * 3), ([4, 4], [0.5, 0.5])], budget=3)
    assert small.n == 3 and [int(x) for x in small.tokens] == [7, 1, 2]   # the best path, ancestors first
    for i in range(1, small.n):
        assert int(small.parents[i]) in range(i)


def test_ancestor_words_and_walk():
    t = build_tree(0, [([1, 2], [1.0, 1.0]), ([3], [0.5])], budget=8)
    w = t.ancestor_words().view(np.uint64)
    for i in range(t.n):
        bits = {j for j in range(t.n) if (int(w[i]) >> j) & 1}
        assert bits == set(t.path(i))
    tok = {int(t.tokens[i]): i for i in range(t.n)}
    picks = [0] * t.n
    picks[0], picks[tok[1]], picks[tok[2]] = 1, 2, 9         # the target agrees with the first chain, then says 9
    path, bonus = walk_greedy(t, picks)
    assert [int(t.tokens[i]) for i in path] == [0, 1, 2] and bonus == 9
    picks[0] = 3                                             # the other branch
    path, bonus = walk_greedy(t, picks)
    assert [int(t.tokens[i]) for i in path] == [0, 3] and bonus == picks[tok[3]]
    picks[0] = 42                                            # no child agrees: only the bonus token
    assert walk_greedy(t, picks) == ([0], 42)
    assert isinstance(t, Tree)
