"""GPU tree construction against the reference's own outputs and the oracle.

Bar: token / depth / parent arrays identical; top-k indices identical;
log-probs and scores within 1e-12 relative (the GPU's log-sum-exp can differ
from numpy's pairwise sum in the last bits). build_tree on the reference's own
top-k arrays is bit-exact in every field, scores included, since it performs
the reference's float64 operations in the reference's order.
"""
import numpy as np
import pytest
import torch

import cast_b200
from cast_b200 import _lib, workloads
from oracle import tree as otree

pytestmark = pytest.mark.gpu

RTOL = 1e-12


def _lp_close(a, b):
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape
    fin = np.isfinite(b)
    assert np.array_equal(np.isfinite(a), fin)
    assert np.all(np.abs(a[fin] - b[fin]) <= RTOL * np.maximum(1.0, np.abs(b[fin])))


def test_block_topk_config1(cuda, golden):
    g = golden("tree_cfg1.npz")
    idx, lp = cast_b200.block_topk(np.random.default_rng(0).normal(scale=5, size=(15, 64)))
    assert np.array_equal(idx, g["idx"])
    _lp_close(lp, g["lp"])


def test_build_tree_config1_bit_exact(cuda, golden):
    g = golden("tree_cfg1.npz")
    for n in (16, 127):
        nodes = cast_b200.build_tree(g["idx"], g["lp"], n)
        assert [nd.token for nd in nodes] == g[f"n{n}_token"].tolist()
        assert [nd.depth for nd in nodes] == g[f"n{n}_depth"].tolist()
        assert [nd.parent for nd in nodes] == g[f"n{n}_parent"].tolist()
        assert np.array_equal(np.array([nd.score for nd in nodes]), g[f"n{n}_score"])


def test_golden_tree_cases(cuda, golden):
    g = golden("tree_cases.npz")
    for name, (seed, L, V, k, budget) in zip(g["names"], g["params"]):
        k, budget = int(k), int(budget)
        idx, lp = cast_b200.block_topk(g[f"{name}_logits"], max(k, 1))
        assert np.array_equal(idx, g[f"{name}_idx"]), name
        _lp_close(lp, g[f"{name}_lp"])
        nodes = cast_b200.build_tree(g[f"{name}_idx"], g[f"{name}_lp"], budget, k)
        assert [nd.token for nd in nodes] == g[f"{name}_token"].tolist(), name
        assert [nd.depth for nd in nodes] == g[f"{name}_depth"].tolist(), name
        assert [nd.parent for nd in nodes] == g[f"{name}_parent"].tolist(), name
        assert np.array_equal(np.array([nd.score for nd in nodes], dtype=np.float64), g[f"{name}_score"]), name


def test_full_vocab_rows(cuda, golden):
    g = golden("topk_vocab.npz")
    for name in ("v151936", "v128256"):
        V = int(name[1:])
        x = np.random.default_rng(list(g[f"{name}_seed"])).normal(scale=5, size=(15, V))
        idx, lp = cast_b200.block_topk(x)
        assert np.array_equal(idx, g[f"{name}_idx"])
        _lp_close(lp, g[f"{name}_lp"])
        nodes = cast_b200.build_tree(idx, lp, 127)
        assert [nd.parent for nd in nodes] == g[f"{name}_n127_parent"].tolist()
        assert [nd.token for nd in nodes] == g[f"{name}_n127_token"].tolist()


@pytest.mark.parametrize("seed", range(12))
def test_random_with_ties_against_oracle(cuda, seed):
    # Every third case rounds the logits to integers: equal log-probs and equal
    # path scores everywhere. There the heap's tie order depends on the last
    # bit of each lp, and numpy's own lse (SIMD exp, pairwise sum) is not
    # reproducible bit for bit across machines; so the tree kernel is checked
    # bit-exact on the lp it was given, and the whole pipeline against the pure
    # oracle on the continuous cases.
    rng = np.random.default_rng(500 + seed)
    B = int(rng.integers(1, 6))
    L = int(rng.integers(1, 16))
    V = int(rng.integers(2, 3000))
    k = int(rng.integers(1, min(V, 24) + 1))
    budget = int(rng.integers(0, 400))
    x = rng.normal(scale=float(rng.choice([0.5, 2.0, 5.0])), size=(B, L, V))
    tied = seed % 3 == 0
    if tied:
        x = np.round(x)
    xd = torch.from_numpy(x).to(cuda)
    idx, lp = cast_b200.block_topk_device(xd, k)
    trees = cast_b200.build_trees(idx, lp, budget, k)
    assert _lib.device_error() == 0
    for b in range(B):
        oi, ol = otree.block_topk(x[b], k)
        gi, gl = idx[b].cpu().numpy(), lp[b].cpu().numpy()
        assert np.array_equal(gi, oi)
        _lp_close(gl, ol)
        n = int(trees.count[b])
        same_lp = otree.build_tree(gi, gl, budget, k)     # the oracle on the GPU's own lp
        assert n == len(same_lp)
        assert np.array_equal(trees.token[b, :n].cpu().numpy(), same_lp.token)
        assert np.array_equal(trees.depth[b, :n].cpu().numpy(), same_lp.depth)
        assert np.array_equal(trees.parent[b, :n].cpu().numpy(), same_lp.parent)
        assert np.array_equal(trees.score[b, :n].cpu().numpy(), same_lp.score)
        if not tied:
            ref = otree.build_tree(oi, ol, budget, k)
            assert np.array_equal(trees.token[b, :n].cpu().numpy(), ref.token)
            assert np.array_equal(trees.parent[b, :n].cpu().numpy(), ref.parent)
            _lp_close(trees.score[b, :n].cpu().numpy(), ref.score)


def test_pack_layout_matches_serving_convention(cuda):
    # the pack arrays of cast_trees/serving.py:213-222, built in the same launch
    w = workloads.Workload("t", 9, 500, [100, 7, 33], [16, 40, 1])
    logits = torch.from_numpy(w.logits_batch()).to(cuda)
    idx, lp = cast_b200.block_topk_device(logits, 8)
    lay = w.layout()
    roots = torch.tensor([3, 4, 5], dtype=torch.int32, device=cuda)
    budget = torch.tensor(w.N, dtype=torch.int32, device=cuda)
    t = cast_b200.build_trees(idx, lp, budget, 8, cu_q=torch.from_numpy(lay["cu_q"]), root_token=roots,
                              seq_len=torch.tensor(w.S, dtype=torch.int32))
    assert _lib.device_error() == 0
    for b in range(w.B):
        oi, ol = otree.block_topk(w.logits(b))
        ref = otree.build_tree(oi, ol, w.N[b])
        q0, q1 = lay["cu_q"][b], lay["cu_q"][b + 1]
        assert t.pack_parent[q0:q1].cpu().tolist() == otree.pack_parent(ref.parent).tolist()
        assert t.pack_token[q0:q1].cpu().tolist() == [3 + b] + ref.token.tolist()
        assert t.pack_pos[q0:q1].cpu().tolist() == [w.S[b]] + (w.S[b] + ref.depth).tolist()


def test_config3_rows_bit_exact(cuda):
    # configuration-3 block scores (V = 128256): GPU tree arrays equal the reference's
    w = workloads.config(3)
    sub = w.shard([0, 1, 2])
    logits = torch.from_numpy(sub.logits_batch()).to(cuda)
    idx, lp = cast_b200.block_topk_device(logits, 8)
    t = cast_b200.build_trees(idx, lp, 127, 8)
    assert _lib.device_error() == 0
    for b in range(sub.B):
        oi, ol = otree.block_topk(sub.logits(b))
        assert np.array_equal(idx[b].cpu().numpy(), oi)
        ref = otree.build_tree(oi, ol, 127)
        assert np.array_equal(t.token[b].cpu().numpy(), ref.token)
        assert np.array_equal(t.parent[b].cpu().numpy(), ref.parent)
        assert np.array_equal(t.depth[b].cpu().numpy(), ref.depth)
        _lp_close(t.score[b].cpu().numpy(), ref.score)


def test_host_argument_errors(cuda):
    x = torch.randn(2, 5, device=cuda, dtype=torch.float64)
    with pytest.raises(_lib.CastError):
        cast_b200.block_topk_device(x, 6)          # k > V
    with pytest.raises(_lib.CastError):
        cast_b200.block_topk_device(x, 0)


@pytest.mark.parametrize("budget, k", [(40, 8), (127, 8), (200, 6)])
def test_tied_logits_pipeline_bit_exact_against_reference(cuda, budget, k):
    # Tie-heavy logits whose log-softmax is exact in both implementations: each row has a single 0
    # (the maximum) and every other logit an integer <= -1000, so every other exp underflows (numpy
    # gives 0; the library's clamped argument adds under 2^-1021, nothing next to the 1), the sum is
    # exactly 1 and lse exactly 0. Every log-prob is then an exact integer, shared by hundreds of
    # tokens, and every path score an exact integer sum: equal scores everywhere, so the tree's order
    # is decided by the (depth, parent, rank) tie rule alone. The whole pipeline from raw logits must
    # match the reference's numpy top-k and heap, bit for bit.
    rng = np.random.default_rng(900 + budget)
    B, L, V = 3, 9, 700
    x = -1000.0 - rng.integers(0, 4, size=(B, L, V)).astype(np.float64)
    x[np.arange(B)[:, None], np.arange(L)[None, :], rng.integers(0, V, size=(B, L))] = 0.0
    xd = torch.from_numpy(x).to(cuda)
    idx, lp = cast_b200.block_topk_device(xd, k)
    trees = cast_b200.build_trees(idx, lp, budget, k)
    assert _lib.device_error() == 0
    for b in range(B):
        oi, ol = otree.block_topk(x[b], k)
        assert np.array_equal(idx[b].cpu().numpy(), oi)
        assert np.array_equal(lp[b].cpu().numpy(), ol)
        ref = otree.build_tree(oi, ol, budget, k)
        n = int(trees.count[b])
        assert n == len(ref)
        assert np.array_equal(trees.token[b, :n].cpu().numpy(), ref.token)
        assert np.array_equal(trees.depth[b, :n].cpu().numpy(), ref.depth)
        assert np.array_equal(trees.parent[b, :n].cpu().numpy(), ref.parent)
        assert np.array_equal(trees.score[b, :n].cpu().numpy().view(np.int64), ref.score.view(np.int64))


@pytest.mark.parametrize("max_budget", [127, 255])
@pytest.mark.parametrize("kind", ["flat", "unsorted", "peaked", "zero_top", "integer_ties", "positive", "one_row"])
def test_build_tree_on_any_rows_bit_exact(cuda, kind, max_budget):
    # build_tree on top-k arrays given directly (not produced by block_topk): rows in any column order,
    # rows whose best lp is 0 or -0.0 (a chain of equal scores), integer lp (ties everywhere), positive
    # lp (children better than their parents). Flat rows take many nodes per batched step, peaked and
    # zero-top rows mostly single pops; every field must equal the reference heap's, score bits included.
    rng = np.random.default_rng(sum(map(ord, kind)) + max_budget)
    B, k = 6, 8
    L = 1 if kind == "one_row" else 15
    idx = rng.integers(0, 128256, size=(B, L, k)).astype(np.int64)
    if kind in ("flat", "unsorted", "one_row"):
        lp = -np.sort(rng.exponential(2.0, size=(B, L, k)), axis=-1) - rng.exponential(1.0, size=(B, L, 1))
    elif kind == "peaked":
        lp = -np.sort(rng.exponential(3.0, size=(B, L, k)), axis=-1)
        lp[..., 0] = -rng.exponential(1e-4, size=(B, L))
    elif kind == "zero_top":
        lp = -np.sort(rng.exponential(2.0, size=(B, L, k)), axis=-1)
        lp[..., 0] = np.where(rng.random((B, L)) < 0.5, 0.0, -0.0)
    elif kind == "integer_ties":
        lp = -np.sort(rng.integers(0, 3, size=(B, L, k)), axis=-1).astype(np.float64)
    else:
        lp = np.sort(rng.normal(0.0, 1.0, size=(B, L, k)), axis=-1)[..., ::-1].copy()
    if kind == "unsorted":
        for b in range(B):
            perm = rng.permutation(k)
            idx[b], lp[b] = idx[b][:, perm], lp[b][:, perm]
    budgets = rng.integers(0, max_budget + 1, size=B).astype(np.int32)
    budgets[0] = max_budget
    trees = cast_b200.build_trees(torch.from_numpy(idx).to(cuda), torch.from_numpy(lp).to(cuda),
                                  torch.from_numpy(budgets).to(cuda), k, max_budget=max_budget)
    assert _lib.device_error() == 0
    for b in range(B):
        ref = otree.build_tree(idx[b], lp[b], int(budgets[b]), k)
        n = int(trees.count[b])
        assert n == len(ref)
        assert np.array_equal(trees.token[b, :n].cpu().numpy(), ref.token)
        assert np.array_equal(trees.depth[b, :n].cpu().numpy(), ref.depth)
        assert np.array_equal(trees.parent[b, :n].cpu().numpy(), ref.parent)
        assert np.array_equal(trees.score[b, :n].cpu().numpy().view(np.int64), ref.score.view(np.int64))
