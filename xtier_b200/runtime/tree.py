"""Multi-branch draft trees for speculative decoding.

Several candidate continuations of one stream -- the draft model's chain, Recall copies from the stream's own context
and from the record -- are merged into one token trie under the last accepted token (the root). The target scores
every node in one forward: node i sits in KV-cache slot `start + i` and at RoPE position `start + depth(i)`, and its
attention sees the cache before `start` plus its own ancestors (a 64-bit ancestor word per node, the tree mask of the
prefill attention kernel). The greedy walk follows, from the root, the child whose token equals the target's pick at
the current node; the accepted nodes' KV is then moved to consecutive slots (`compact`). With greedy targets the
output is exactly the target's own greedy continuation: every accepted token is the target's pick after its accepted
prefix.

Nodes are kept by expected acceptance -- the product of the candidates' per-token confidences along the path (1 for
a copy, the draft probability for a draft token) -- under a node budget, always with their ancestors, in breadth-first
order (parents before children).

Reference parity: xtier/packs/deepseek_v4/recall/tree.py:110-300, 386-433 (candidates merged into one trie under the
verified token, a node budget, the ancestor mask, the greedy walk). The trie, scoring and layout here are this
project's own; sampling verification of trees (SpecInfer) is not built: trees are verified greedily.
"""
from __future__ import annotations

import dataclasses

import numpy as np

MAX_NODES = 64   # one 64-bit ancestor word per node


@dataclasses.dataclass
class Tree:
    tokens: np.ndarray      # int64 [n]; node 0 is the root (the last accepted token)
    parents: np.ndarray     # int32 [n]; -1 for the root, else an earlier node
    depth: np.ndarray       # int32 [n]
    score: np.ndarray       # float64 [n]: expected acceptance of the path to the node

    @property
    def n(self) -> int:
        return int(self.tokens.shape[0])

    def children(self, i: int) -> list[int]:
        return [int(c) for c in np.nonzero(self.parents == i)[0]]

    def ancestor_words(self) -> np.ndarray:
        """int64 [n]: bit j of word i is set when node j is node i or one of its ancestors."""
        words = np.zeros(self.n, np.uint64)
        for i in range(self.n):
            p = int(self.parents[i])
            words[i] = (words[p] if p >= 0 else np.uint64(0)) | np.uint64(1 << i)
        return words.view(np.int64)

    def path(self, i: int) -> list[int]:
        out = []
        while i >= 0:
            out.append(i)
            i = int(self.parents[i])
        return out[::-1]


def build_tree(root: int, chains, budget: int = 16) -> Tree:
    """Merges candidate chains [(tokens, confidences)] under `root` into a trie of at most `budget` nodes (root
    included, <= 64): the nodes of highest expected acceptance with all their ancestors, breadth-first."""
    budget = max(1, min(int(budget), MAX_NODES))
    tok, par, sc = [int(root)], [-1], [1.0]
    kids: dict = {}
    for toks, conf in chains:
        cur, s = 0, 1.0
        for t, c in zip(toks, conf):
            s *= float(min(max(c, 0.0), 1.0))
            key = (cur, int(t))
            if key in kids:
                cur = kids[key]
                sc[cur] = max(sc[cur], s)
            else:
                tok.append(int(t))
                par.append(cur)
                sc.append(s)
                kids[key] = cur = len(tok) - 1
    n = len(tok)
    par_a, sc_a = np.asarray(par), np.asarray(sc)
    # scores never grow along a path (confidences <= 1), so the best nodes with their ancestors fit the budget
    # when ties go to shallower nodes
    depth = np.zeros(n, np.int32)
    for i in range(1, n):
        depth[i] = depth[par_a[i]] + 1
    order = sorted(range(n), key=lambda i: (-sc_a[i], depth[i], i))
    keep: set = set()
    for i in order:
        if len(keep) >= budget:
            break
        chain = []
        j = i
        while j >= 0 and j not in keep:
            chain.append(j)
            j = int(par_a[j])
        if len(keep) + len(chain) <= budget:
            keep.update(chain)
    kept = sorted(keep, key=lambda i: (depth[i], i))   # breadth-first: parents before children
    new = {old: k for k, old in enumerate(kept)}
    return Tree(np.asarray([tok[i] for i in kept], np.int64),
                np.asarray([new[int(par_a[i])] if par_a[i] >= 0 else -1 for i in kept], np.int32),
                np.asarray([depth[i] for i in kept], np.int32), np.asarray([sc_a[i] for i in kept], np.float64))


def walk_greedy(tree: Tree, picks) -> tuple[list[int], int]:
    """(accepted node indices from the root, the bonus token): from the root, follow the child whose token is the
    target's pick at the current node; the pick at the last accepted node is the bonus token."""
    picks = [int(p) for p in picks]
    cur, path = 0, [0]
    while True:
        nxt = [c for c in tree.children(cur) if int(tree.tokens[c]) == picks[cur]]
        if not nxt:
            return path, picks[cur]
        cur = nxt[0]
        path.append(cur)
