"""CPU check of the GPU tree builder's algorithm against the reference heap.

The build_tree kernel keeps, per expanded node, only its next unpopped child
(children ordered by (neg_child, rank)) and compares keys as ordered 64-bit
patterns. This file restates that scheme in Python and checks that it pops
exactly the reference's nodes (oracle.tree.build_tree, itself pinned to the
reference) on random inputs, including inputs full of ties.
"""
import struct

import numpy as np
import pytest

from oracle import tree as otree


def ordered_key(v):
    u = struct.unpack("<Q", struct.pack("<d", v + 0.0))[0]
    return (~u) & 0xFFFFFFFFFFFFFFFF if u >> 63 else u | (1 << 63)


def lazy_build(top_idx, top_lp, budget, k=8):
    L = top_idx.shape[0]
    k = min(k, top_idx.shape[1])
    lp = np.asarray(top_lp, dtype=np.float64)

    def order(base, d, root):
        keys = [(ordered_key(-float(lp[0, r]) if root else base - float(lp[d, r])), r) for r in range(k)]
        return [r for _, r in sorted(keys)]

    orders = {-1: order(0.0, 0, True)}
    node_neg = []
    cand = []  # (hi, lo, neg, parent, j, depth, rank)
    if budget > 0 and k > 0:
        r = orders[-1][0]
        neg = -float(lp[0, r])
        cand.append((ordered_key(neg), (1 << 40) | r, neg, -1, 0, 1, r))
    tok, dep, par, sc = [], [], [], []
    while len(tok) < budget and cand:
        s = min(range(len(cand)), key=lambda c: (cand[c][0], cand[c][1]))
        _, _, neg, p, j, d, r = cand[s]
        me = len(tok)
        tok.append(int(top_idx[d - 1, r])); dep.append(d); par.append(p); sc.append(-neg)
        node_neg.append(neg)
        if j + 1 < k:
            r2 = orders[p][j + 1]
            sneg = -float(lp[0, r2]) if p < 0 else node_neg[p] - float(lp[d - 1, r2])
            cand[s] = (ordered_key(sneg), (d << 40) | ((p + 1) << 8) | r2, sneg, p, j + 1, d, r2)
        else:
            cand[s] = cand[-1]
            cand.pop()
        if d < L:
            orders[me] = order(neg, d, False)
            r2 = orders[me][0]
            cneg = neg - float(lp[d, r2])
            cand.append((ordered_key(cneg), ((d + 1) << 40) | ((me + 1) << 8) | r2, cneg, me, 0, d + 1, r2))
    return tok, dep, par, sc


def _check(idx, lp, budget, k):
    ref = otree.build_tree(idx, lp, budget, k)
    tok, dep, par, sc = lazy_build(idx, lp, budget, k)
    assert tok == ref.token.tolist()
    assert dep == ref.depth.tolist()
    assert par == ref.parent.tolist()
    assert np.array_equal(np.array(sc, dtype=np.float64), ref.score)


def test_lazy_matches_reference_on_golden_cases(golden):
    g = golden("tree_cases.npz")
    for name, (seed, L, V, k, budget) in zip(g["names"], g["params"]):
        _check(g[f"{name}_idx"], g[f"{name}_lp"], int(budget), int(k))


@pytest.mark.parametrize("seed", range(40))
def test_lazy_matches_reference_random_ties(seed):
    rng = np.random.default_rng(1000 + seed)
    L = int(rng.integers(1, 16))
    V = int(rng.integers(2, 60))
    k = int(rng.integers(1, min(V, 12) + 1))
    budget = int(rng.integers(0, 300))
    x = rng.normal(scale=float(rng.choice([0.0, 0.5, 2.0, 5.0])), size=(L, V))
    if seed % 2 == 0:
        x = np.round(x * 2) / 2          # many exact ties
    idx, lp = otree.block_topk(x, k)
    _check(idx, lp, budget, k)


def test_lazy_matches_reference_unsorted_rows():
    # build_tree accepts any (L, k) arrays, not only sorted block_topk output
    rng = np.random.default_rng(7)
    for _ in range(20):
        L, k = int(rng.integers(1, 10)), int(rng.integers(1, 9))
        lp = -np.abs(np.round(rng.normal(size=(L, k)), 1))
        idx = rng.integers(0, 1000, size=(L, k))
        _check(idx, lp, int(rng.integers(1, 120)), k)


def test_negative_zero_ties():
    # lp of exactly 0.0 gives neg = -0.0; Python treats -0.0 == 0.0 as a tie
    lp = np.array([[0.0, -0.0, -1.0], [-0.0, 0.0, -2.0], [0.0, -1e-300, -0.0]])
    idx = np.arange(9).reshape(3, 3)
    _check(idx, lp, 20, 3)
