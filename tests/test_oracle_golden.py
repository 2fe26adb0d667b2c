"""The CPU oracle against the reference's own outputs (tests/golden/*.npz)."""
import numpy as np
import pytest
import torch

from oracle import attn as oattn
from oracle import tree as otree
from tests.golden.make_golden import ragged_scenario


def test_block_topk_config1_bit_exact(golden):
    g = golden("tree_cfg1.npz")
    idx, lp = otree.block_topk(np.random.default_rng(0).normal(scale=5, size=(15, 64)))
    assert np.array_equal(idx, g["idx"])
    assert np.array_equal(lp, g["lp"])          # bit-exact float64


@pytest.mark.parametrize("n", [16, 127])
def test_build_tree_config1(golden, n):
    g = golden("tree_cfg1.npz")
    t = otree.build_tree(g["idx"], g["lp"], n)
    for key in ("token", "depth", "parent", "score"):
        assert np.array_equal(getattr(t, key), g[f"n{n}_{key}"]), key
    assert otree.expected_accepted_length(t) == g[f"n{n}_expected_len"]


def test_config1_tree_head_and_quickstart_pin(golden):
    g = golden("tree_cfg1.npz")
    t = otree.build_tree(g["idx"], g["lp"], 16)
    head = list(zip(t.token[:6], t.depth[:6], t.parent[:6]))
    assert head == [(47, 1, -1), (15, 2, 0), (48, 1, -1), (62, 1, -1), (36, 3, 1), (27, 4, 4)]
    t127 = otree.build_tree(g["idx"], g["lp"], 127)
    assert f"{otree.expected_accepted_length(t127):.2f}" == "3.54"   # README quickstart line


def test_build_tree_cases(golden):
    g = golden("tree_cases.npz")
    for name, (seed, L, V, k, budget) in zip(g["names"], g["params"]):
        idx, lp = otree.block_topk(g[f"{name}_logits"], max(int(k), 1))
        assert np.array_equal(idx, g[f"{name}_idx"]), name
        assert np.array_equal(lp, g[f"{name}_lp"]), name
        t = otree.build_tree(idx, lp, int(budget), int(k))
        for key in ("token", "depth", "parent", "score"):
            assert np.array_equal(getattr(t, key), g[f"{name}_{key}"]), (name, key)


def test_block_topk_full_vocab(golden):
    g = golden("topk_vocab.npz")
    for name in ("v151936", "v128256"):
        V = int(name[1:])
        x = np.random.default_rng(list(g[f"{name}_seed"])).normal(scale=5, size=(15, V))
        idx, lp = otree.block_topk(x)
        assert np.array_equal(idx, g[f"{name}_idx"])
        assert np.array_equal(lp, g[f"{name}_lp"])
        t = otree.build_tree(idx, lp, 127)
        assert np.array_equal(t.parent, g[f"{name}_n127_parent"])
        assert np.array_equal(t.token, g[f"{name}_n127_token"])


def test_ancestor_words_match_reference_bits():
    sc = ragged_scenario()
    cu = sc["cu_q"].numpy()
    for b, (S, P, parent) in enumerate(sc["reqs"]):
        w = otree.ancestor_words(np.array(parent))
        assert w.shape == (P, 1)
        assert np.array_equal(w[:, 0].view(np.int64), sc["bits"][cu[b]:cu[b] + P])


def test_ancestor_words_multiword():
    rng = np.random.default_rng(3)
    P = 200
    parent = np.array([-1] + [int(rng.integers(0, i)) for i in range(1, P)])
    w = otree.ancestor_words(parent)
    vis = otree.ancestor_matrix_from_parent(parent)
    for i in range(P):
        for j in range(P):
            assert bool((int(w[i, j // 64]) >> (j % 64)) & 1) == vis[i, j]


def test_attention_config1_matches_reference_sdpa(golden):
    g = golden("attn_cfg1.npz")
    S, P = int(g["S"]), int(g["P"])
    gen = torch.Generator().manual_seed(0)
    q = torch.randn(P, 32, 128, generator=gen)
    k = torch.randn(S + P, 8, 128, generator=gen)
    v = torch.randn(S + P, 8, 128, generator=gen)
    words = otree.ancestor_words(otree.pack_parent(g["parent"]))
    out = oattn.tree_attention(q, k, v, [0, P], [0, S + P], [S], [P], [words])
    err = (out - torch.from_numpy(g["out"])).abs().max().item()
    assert err < 1e-5, err


def test_attention_ragged_matches_reference(golden):
    g = golden("attn_ragged.npz")
    sc = ragged_scenario(int(g["seed"]))
    out = oattn.tree_attention(sc["q"], sc["k"], sc["v"], sc["cu_q"], sc["cu_kv"], sc["prefix"],
                               sc["pack"], sc["bits"])
    err = (out - torch.from_numpy(g["out"])).abs().max().item()
    assert err < 1e-5, err


def test_attention_empty_rows_are_zero():
    # a pack row with no prefix and no visible pack key returns 0 (tree_attn.py:89)
    q = torch.randn(2, 4, 16)
    k = torch.randn(2, 2, 16)
    v = torch.randn(2, 2, 16)
    bits = np.array([0, 3], dtype=np.int64)
    out = oattn.tree_attention(q, k, v, [0, 2], [0, 2], [0], [2], bits)
    assert torch.all(out[0] == 0)
    assert torch.all(torch.isfinite(out))


def test_walk_tree_greedy(golden):
    g = golden("walk.npz")
    for c in range(6):
        path, bonus = otree.walk_tree_greedy(g[f"c{c}_parent"], g[f"c{c}_token"], g[f"c{c}_logits"])
        assert path == g[f"c{c}_path"].tolist()
        assert bonus == int(g[f"c{c}_bonus"])


def _forest(g, prefix):
    cnt = g[prefix + "count"]
    return [otree.Tree(g[prefix + "token"][b, :n], g[prefix + "depth"][b, :n], g[prefix + "parent"][b, :n],
                       g[prefix + "score"][b, :n]) for b, n in enumerate(cnt)]


@pytest.mark.parametrize("forest", ["rand", "ties", "same"])
def test_select_global_topk(golden, forest):
    g = golden("select.npz")
    trees = _forest(g, f"{forest}_in_")
    for total in g["totals"].tolist():
        got = otree.select_global_topk(trees, total)
        want = _forest(g, f"{forest}_t{total}_")
        assert [len(t) for t in got] == [len(t) for t in want], total
        for a, b in zip(got, want):
            for f in ("token", "depth", "parent"):
                assert np.array_equal(getattr(a, f), getattr(b, f)), (total, f)
            assert np.array_equal(a.score, b.score)


@pytest.mark.parametrize("case", ["inplace", "compact", "grow"])
def test_append_store(golden, case):
    from oracle import kv as okv
    g = golden("append.npz")
    keep = [[int(x) for x in row if x >= 0] for row in g[f"{case}_keep"]]
    ks, vs, new_len = okv.append_store(list(g[f"{case}_in_k"]), list(g[f"{case}_in_v"]),
                                       g[f"{case}_store_len"].tolist(), g[f"{case}_cu_q"].tolist(), keep,
                                       g[f"{case}_accepted"].tolist(), g[f"{case}_rows"].tolist(),
                                       list(g[f"{case}_pack_k"]), list(g[f"{case}_pack_v"]))
    assert new_len == g[f"{case}_new_len"].tolist()
    assert np.array_equal(np.stack(ks), g[f"{case}_out_k"])
    assert np.array_equal(np.stack(vs), g[f"{case}_out_v"])


def test_gather_cache(golden):
    from oracle import kv as okv
    g = golden("gather.npz")
    ks, vs = okv.gather_cache(list(g["in_k"]), list(g["in_v"]), int(g["n_prefix"]), g["keep"].tolist())
    assert np.array_equal(np.stack(ks), g["out_k"])
    assert np.array_equal(np.stack(vs), g["out_v"])
