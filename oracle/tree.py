"""CPU oracle for best-first tree construction (test infrastructure only).

Each function cites the reference lines it restates. ``block_topk`` keeps the
reference's numpy operation sequence on purpose: the GPU kernel is checked
bit-exact against it, so the oracle has to produce exactly the reference's
float64 values (pinned by tests/golden/tree_*.npz, made by the reference).
"""
import heapq
from typing import NamedTuple

import numpy as np


class Tree(NamedTuple):
    """One best-first tree in pop order (cast_trees/tree.py:12-17 as arrays)."""
    token: np.ndarray   # int64 [N]
    depth: np.ndarray   # int64 [N], 1..L
    parent: np.ndarray  # int64 [N], -1 = root, else index < own index
    score: np.ndarray   # float64 [N], path log-probability

    def __len__(self):
        return int(self.token.shape[0])


def block_topk(logits, k=8):
    """fp64 log-softmax per row, then the k best by a stable descending sort.

    Restates cast_trees/tree.py:20-26. Ties keep the lower vocabulary index
    first (argsort of the negated values with kind="stable").
    """
    x = np.asarray(logits, dtype=np.float64)
    shifted = x - x.max(axis=-1, keepdims=True)
    lse = np.log(np.exp(shifted).sum(axis=-1, keepdims=True))
    lp = shifted - lse
    order = np.argsort(-lp, axis=-1, kind="stable")[..., :k]
    return order, np.take_along_axis(lp, order, axis=-1)


def build_tree(top_idx, top_lp, budget, k=8):
    """Best-first prefix-closed tree with `budget` non-root nodes.

    Restates cast_trees/tree.py:29-49: a min-heap on the key
    (-path_logprob, depth, parent, rank, push counter); every pop appends a
    node and pushes its k children (if depth < L). Path scores are formed
    with the same float64 operation order: -lp[0, r] for depth 1 and
    neg_parent - lp[d, r] below it.
    """
    top_idx = np.asarray(top_idx)
    top_lp = np.asarray(top_lp, dtype=np.float64)
    L = top_idx.shape[0]
    k = min(k, top_idx.shape[1])
    heap = []
    serial = 0
    for r in range(k):
        heap.append((-float(top_lp[0, r]), 1, -1, r, serial))
        serial += 1
    heapq.heapify(heap)
    tok, dep, par, sc = [], [], [], []
    while heap and len(tok) < budget:
        neg, d, p, r, _ = heapq.heappop(heap)
        me = len(tok)
        tok.append(int(top_idx[d - 1, r]))
        dep.append(d)
        par.append(p)
        sc.append(-neg)
        if d < L:
            for r2 in range(k):
                heapq.heappush(heap, (neg - float(top_lp[d, r2]), d + 1, me, r2, serial))
                serial += 1
    return Tree(np.array(tok, dtype=np.int64), np.array(dep, dtype=np.int64),
                np.array(par, dtype=np.int64), np.array(sc, dtype=np.float64))


def expected_accepted_length(tree):
    """Sum of path masses, cast_trees/tree.py:58-60 (left-to-right float sum)."""
    total = 0.0
    for s in tree.score:
        total += float(np.exp(s))
    return total


def pack_parent(tree_parent):
    """Pack-local parent array: [root] + nodes, node i at pack index i+1.

    Convention of cast_trees/serving.py:217-222 (packed parent = parent + 1,
    root parent = -1).
    """
    tree_parent = np.asarray(tree_parent, dtype=np.int64)
    return np.concatenate([[-1], tree_parent + 1]).astype(np.int32)


def ancestor_matrix_from_parent(parent):
    """(P, P) bool, row i marks i and its ancestors (cast_trees/tree.py:85-93)."""
    parent = np.asarray(parent)
    P = parent.shape[0]
    vis = np.zeros((P, P), dtype=bool)
    for i in range(P):
        if parent[i] >= 0:
            vis[i] = vis[parent[i]]
        vis[i, i] = True
    return vis


def ancestor_words(parent, words=None):
    """Ancestor bitsets as little-endian uint64 words, [P, W].

    Bit j of row i is set iff pack token j is i or an ancestor of i. With one
    word this is the int64 mask of cast_trees/serving.py:218-222 and
    tests/test_tree_attn.py:22-27.
    """
    vis = ancestor_matrix_from_parent(parent)
    P = vis.shape[0]
    W = (P + 63) // 64 if words is None else words
    out = np.zeros((P, W), dtype=np.uint64)
    for i in range(P):
        for j in np.nonzero(vis[i])[0]:
            out[i, j // 64] |= np.uint64(1) << np.uint64(j % 64)
    return out


def walk_tree_greedy(parent, token, logits):
    """Greedy tree walk, cast_trees/decode.py:85-103 at temperature 0.

    parent/token: the tree's node arrays (tree-local parent, -1 = root).
    logits: [1+N, V] target logits of the packed rows. Returns (path, bonus):
    path = accepted node indices, bonus = the token picked after the path.
    """
    children = {i: [] for i in range(-1, len(parent))}
    for i, p in enumerate(parent):
        children[int(p)].append(i)
    path, cur = [], -1
    while True:
        pick = int(np.argmax(logits[cur + 1]))
        hit = next((c for c in children[cur] if int(token[c]) == pick), None)
        if hit is None:
            return path, pick
        path.append(hit)
        cur = hit


def select_global_topk(trees, total):
    """Shared-budget split of a forest, cast_trees/tree.py:63-82.

    trees: list of Tree. The pool of (score, tree, node) is ordered by
    (-score, tree, node) - Python's sort, so -0.0 and 0.0 tie - and the first
    `total` entries (Python slice semantics, negative totals included) are
    kept; each tree keeps its nodes in order and parents are renumbered, -1
    where the parent was not kept.
    """
    pool = [(float(t.score[j]), b, j) for b, t in enumerate(trees) for j in range(len(t))]
    pool.sort(key=lambda e: (-e[0], e[1], e[2]))
    keep = [set() for _ in trees]
    for _, b, j in pool[:total]:
        keep[b].add(j)
    out = []
    for b, t in enumerate(trees):
        kept = sorted(keep[b])
        remap = {-1: -1}
        for new, old in enumerate(kept):
            remap[old] = new
        idx = np.array(kept, dtype=np.int64)
        out.append(Tree(t.token[idx].astype(np.int64), t.depth[idx].astype(np.int64),
                        np.array([remap.get(int(t.parent[i]), -1) for i in kept], dtype=np.int64),
                        t.score[idx].astype(np.float64)))
    return out
