"""The verify-round steps around attention on the GPU: greedy walk, global
top-k selection, KV-store append and cache gather.

Each is checked bit-exact against the reference's own outputs
(tests/golden/walk.npz, select.npz, append.npz, gather.npz) and against the
CPU oracle on larger seeded cases and the edge cases the reference's code
paths have (ties, compaction, growth, empty paths, NaN / -inf logits).
"""
import types

import numpy as np
import pytest
import torch

import cast_b200
from cast_b200 import _lib
from oracle import kv as okv
from oracle import tree as otree

pytestmark = pytest.mark.gpu


# ----------------------------------------------------------------------------- walk
def test_walk_tree_matches_reference_golden(cuda, golden):
    g = golden("walk.npz")
    for c in range(6):
        parent, token = g[f"c{c}_parent"], g[f"c{c}_token"]
        logits = g[f"c{c}_logits"].astype(np.float32)
        # fp32 rounding keeps the reference's choices (margins are large)
        assert otree.walk_tree_greedy(parent, token, logits) == (g[f"c{c}_path"].tolist(), int(g[f"c{c}_bonus"]))
        nodes = [cast_b200.TreeNode(int(t), 1, int(p), 0.0) for t, p in zip(token, parent)]
        path, bonus = cast_b200.walk_tree(nodes, torch.from_numpy(logits).to(cuda))
        assert path == g[f"c{c}_path"].tolist() and bonus == int(g[f"c{c}_bonus"])


def _walk_case(seed, B, V, n_nodes, dtype, follow=0.85, dev="cuda"):
    """GPU trees for B sequences and logits that follow each tree for a while."""
    rng = np.random.default_rng(seed)
    block = torch.from_numpy(rng.normal(scale=3.0, size=(B, 15, min(V, 64)))).to(dev)
    idx, lp = cast_b200.block_topk_device(block, 8)
    P = [n_nodes + 1] * B
    cu_q = np.concatenate([[0], np.cumsum(P)]).astype(np.int32)
    root = torch.from_numpy(rng.integers(0, V, size=B).astype(np.int32)).to(dev)
    trees = cast_b200.build_trees(idx, lp, n_nodes, 8, cu_q=torch.from_numpy(cu_q).to(dev), root_token=root,
                                  total_q=int(cu_q[-1]))
    parent = trees.pack_parent.cpu().numpy()
    token = trees.pack_token.cpu().numpy()
    logits = rng.normal(size=(int(cu_q[-1]), V)).astype(np.float32)
    for b in range(B):
        q0 = cu_q[b]
        for r in range(P[b]):
            kids = [c for c in range(r + 1, P[b]) if parent[q0 + c] == r]
            if kids and rng.random() < follow:
                logits[q0 + r, token[q0 + kids[int(rng.integers(len(kids)))]]] += 8.0
    lt = torch.from_numpy(logits).to(dev, dtype)
    return cu_q, parent, token, lt


def _check_walk(w, cu_q, parent, token, logits_host):
    B = len(cu_q) - 1
    acc = w.accepted.cpu().numpy()
    path = w.path.cpu().numpy()
    bonus = w.bonus.cpu().numpy()
    keep = w.keep.cpu().numpy()
    toks = w.tokens.cpu().numpy()
    lengths = []
    for b in range(B):
        q0, q1 = cu_q[b], cu_q[b + 1]
        tree_parent = parent[q0 + 1:q1] - 1
        p_ref, bonus_ref = otree.walk_tree_greedy(tree_parent, token[q0 + 1:q1], logits_host[q0:q1])
        n = len(p_ref)
        assert acc[b] == n + 1
        assert path[b, :n].tolist() == p_ref and (path[b, n:] == -1).all()
        assert bonus[b] == bonus_ref
        assert keep[b, :n + 1].tolist() == [0] + [i + 1 for i in p_ref] and (keep[b, n + 1:] == -1).all()
        assert toks[b, :n + 1].tolist() == [int(token[q0 + 1 + i]) for i in p_ref] + [bonus_ref]
        lengths.append(n + 1)
    return lengths


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_walk_batched_vs_oracle(cuda, dtype):
    B, V, n = 64, 128256, 127
    cu_q, parent, token, lt = _walk_case(1, B, V, n, dtype)
    w = cast_b200.walk_trees_greedy(lt, torch.from_numpy(cu_q).to(cuda), parent, token, n)
    assert _lib.device_error() == 0
    lengths = _check_walk(w, cu_q, parent, token, lt.float().cpu().numpy())
    assert max(lengths) >= 4 and min(lengths) <= 3


@pytest.mark.parametrize("B", [1, 3, 300])
def test_walk_cluster_sizes_and_odd_vocab(cuda, B):
    # B = 1 / 3 run 8-CTA clusters, B = 300 single CTAs; V = 1001 leaves a scalar tail
    cu_q, parent, token, lt = _walk_case(2 + B, B, 1001, 20, torch.bfloat16)
    w = cast_b200.walk_trees_greedy(lt, torch.from_numpy(cu_q).to(cuda), parent, token, 20)
    assert _lib.device_error() == 0
    _check_walk(w, cu_q, parent, token, lt.float().cpu().numpy())


def test_walk_unaligned_rows_ties_nan_and_single_node(cuda):
    V = 517
    rng = np.random.default_rng(9)
    # three packs: a one-row pack, a chain, a star
    parent = np.array([-1, -1, 0, 1, 2, -1, 0, 0, 0], dtype=np.int32)
    token = np.array([5, 7, 3, 4, 9, 1, 10, 11, 10], dtype=np.int32)
    cu_q = np.array([0, 1, 5, 9], dtype=np.int32)
    logits = rng.normal(size=(9, V)).astype(np.float32)
    logits[0, 200] = 50.0                       # one-row pack: bonus 200
    logits[1, [3, 8]] = 40.0                    # tie: the lower index (3) wins and matches node 1
    logits[2, 4] = float("inf")                 # +inf is a value like any other
    logits[3, :] = -float("inf")                # all -inf: argmax 0 (miss, bonus 0)
    logits[5, 10] = 30.0                        # star: token 10 at pack rows 1 and 3: lowest row wins
    logits[6, 77] = float("nan")                # NaN beats everything: bonus 77
    logits[6, 12] = float("nan")                # ... and the first NaN wins: 12
    store = np.zeros((9, V + 1), dtype=np.float32)   # row stride V + 1: no 16-byte vector path
    store[:, :V] = logits
    lt = torch.from_numpy(store).to(cuda)[:, :V]
    w = cast_b200.walk_trees_greedy(lt, torch.from_numpy(cu_q).to(cuda), parent, token, 4)
    assert _lib.device_error() == 0
    _check_walk(w, cu_q, parent, token, logits)
    assert w.bonus.cpu().tolist() == [200, 0, 12]


def test_walk_path_overflow_is_reported(cuda):
    parent = np.array([-1, 0, 1, 2], dtype=np.int32)
    token = np.array([0, 1, 2, 3], dtype=np.int32)
    logits = np.zeros((4, 8), dtype=np.float32)
    for r in range(3):
        logits[r, r + 1] = 5.0
    w = cast_b200.walk_trees_greedy(torch.from_numpy(logits).to(cuda), torch.tensor([0, 4], device=cuda),
                                    parent, token, 2)
    assert _lib.device_error() == _lib.CAST_DEV_TREE_OVERFLOW
    assert int(w.accepted[0]) == 0 and int(w.bonus[0]) == -1


# --------------------------------------------------------------------------- select
def _golden_forest(g, prefix):
    cnt = g[prefix + "count"]
    return [[cast_b200.TreeNode(int(g[prefix + "token"][b, j]), int(g[prefix + "depth"][b, j]),
                                int(g[prefix + "parent"][b, j]), float(g[prefix + "score"][b, j]))
             for j in range(n)] for b, n in enumerate(cnt)]


@pytest.mark.parametrize("forest", ["rand", "ties", "same"])
def test_select_global_topk_matches_reference_golden(cuda, golden, forest):
    g = golden("select.npz")
    trees = _golden_forest(g, f"{forest}_in_")
    for total in g["totals"].tolist():
        got = cast_b200.select_global_topk(trees, total)
        want = _golden_forest(g, f"{forest}_t{total}_")
        assert got == want, (forest, total)


def test_select_device_pack_layout_vs_oracle(cuda):
    rng = np.random.default_rng(5)
    B, w = 64, 48
    block = torch.from_numpy(rng.normal(scale=5.0, size=(B, 15, 300))).to(cuda)
    idx, lp = cast_b200.block_topk_device(block, 8)
    trees = cast_b200.build_trees(idx, lp, w, 8)
    root = rng.integers(0, 300, size=B).astype(np.int32)
    seq = rng.integers(100, 5000, size=B).astype(np.int32)
    total = B * 8
    sel = cast_b200.select_global_topk_device(trees, total, root_token=root, seq_len=seq)
    assert _lib.device_error() == 0
    host = [otree.Tree(*(x[b, :w].cpu().numpy().astype(np.float64 if x.dtype == torch.float64 else np.int64)
                         for x in (trees.token, trees.depth, trees.parent, trees.score))) for b in range(B)]
    ref = otree.select_global_topk(host, total)
    cnt = sel.count.cpu().numpy()
    assert cnt.sum() == total and cnt.tolist() == [len(t) for t in ref]
    cu = sel.cu_q.cpu().numpy()
    assert cu.tolist() == np.concatenate([[0], np.cumsum(1 + cnt)]).tolist()
    pp, pt, ppos = (x.cpu().numpy() for x in (sel.pack_parent, sel.pack_token, sel.pack_pos))
    for b, t in enumerate(ref):
        n = len(t)
        assert sel.token[b, :n].cpu().numpy().tolist() == t.token.tolist()
        assert sel.parent[b, :n].cpu().numpy().tolist() == t.parent.tolist()
        assert np.array_equal(sel.score[b, :n].cpu().numpy(), t.score)
        q0 = cu[b]
        assert pp[q0:q0 + n + 1].tolist() == [-1] + (t.parent + 1).tolist()
        assert pt[q0:q0 + n + 1].tolist() == [root[b]] + t.token.tolist()
        assert ppos[q0:q0 + n + 1].tolist() == [seq[b]] + (seq[b] + t.depth).tolist()
    # the selected trees stay prefix-closed (cast_trees/tree.py:66-67)
    for t in ref:
        for i in range(len(t)):
            assert -1 <= t.parent[i] < i


# ---------------------------------------------------------------------- append store
def _append_inputs(g, case, dev, dtype=torch.float32):
    to = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev, dtype)
    keep = [[int(x) for x in row if x >= 0] for row in g[f"{case}_keep"]]
    return ([to(x) for x in g[f"{case}_in_k"]], [to(x) for x in g[f"{case}_in_v"]],
            g[f"{case}_store_len"].tolist(), g[f"{case}_cu_q"].tolist(), keep, g[f"{case}_accepted"].tolist(),
            g[f"{case}_rows"].tolist(), [to(x) for x in g[f"{case}_pack_k"]], [to(x) for x in g[f"{case}_pack_v"]])


@pytest.mark.parametrize("case", ["inplace", "compact", "grow"])
def test_append_store_matches_reference_golden(cuda, golden, case):
    g = golden("append.npz")
    args = _append_inputs(g, case, cuda)
    in_ptr = args[0][0].data_ptr()
    ks, vs, new_len = cast_b200.append_store(*args)
    assert _lib.device_error() == 0
    assert new_len == g[f"{case}_new_len"].tolist()
    assert np.array_equal(torch.stack(ks).cpu().numpy(), g[f"{case}_out_k"])
    assert np.array_equal(torch.stack(vs).cpu().numpy(), g[f"{case}_out_v"])
    # in place exactly when the reference keeps its tensors (no drop, no growth)
    assert (ks[0].data_ptr() == in_ptr) == (case == "inplace")


@pytest.mark.parametrize("rows", ["all", "drop"])
def test_append_store_bf16_strided_pack_vs_oracle(cuda, rows):
    rng = np.random.default_rng(12)
    L, B, H, cap, D = 4, 6, 8, 300, 128
    sl = rng.integers(0, 200, size=B).tolist()
    P = rng.integers(2, 40, size=B).tolist()
    cu_q = np.concatenate([[0], np.cumsum(P)]).tolist()
    keep, acc = [], []
    for b in range(B):
        path = sorted(rng.choice(np.arange(1, P[b]), size=int(rng.integers(0, min(P[b] - 1, 12) + 1)),
                             replace=False).tolist())
        keep.append([0] + path)
        acc.append(len(path) + 1)
    bufk = [torch.randn(B, H, cap, D, device=cuda).to(torch.bfloat16) for _ in range(L)]
    bufv = [torch.randn(B, H, cap, D, device=cuda).to(torch.bfloat16) for _ in range(L)]
    # pack K/V as the hook hands them over: key[0] of a [1, H, T, D] tensor made by a transpose
    pk = [torch.randn(1, cu_q[-1], H, D, device=cuda).to(torch.bfloat16).transpose(1, 2)[0] for _ in range(L)]
    pv = [torch.randn(1, cu_q[-1], H, D, device=cuda).to(torch.bfloat16).transpose(1, 2)[0] for _ in range(L)]
    keep_rows = list(range(B)) if rows == "all" else [0, 2, 3, 5]
    host = lambda ts: [t.float().cpu().numpy() for t in ts]
    rk, rv, rlen = okv.append_store(host(bufk), host(bufv), sl, cu_q, keep, acc, keep_rows, host(pk), host(pv))
    ks, vs, new_len = cast_b200.append_store(bufk, bufv, sl, cu_q, keep, acc, keep_rows, pk, pv)
    assert _lib.device_error() == 0
    assert new_len == rlen
    for li in range(L):
        assert np.array_equal(ks[li].float().cpu().numpy(), rk[li])
        assert np.array_equal(vs[li].float().cpu().numpy(), rv[li])


def test_append_store_inplace_from_walk(cuda):
    # the all-device round: walk -> keep rows -> in-place append, no host lists
    B, V, n = 16, 4096, 31
    cu_q, parent, token, lt = _walk_case(3, B, V, n, torch.bfloat16)
    cu_t = torch.from_numpy(cu_q).to(cuda)
    w = cast_b200.walk_trees_greedy(lt, cu_t, parent, token, n)
    L, H, cap, D = 2, 8, 512, 128
    sl = torch.randint(0, 400, (B,), dtype=torch.int32, device=cuda)
    bufk = [torch.randn(B, H, cap, D, device=cuda).to(torch.bfloat16) for _ in range(L)]
    bufv = [torch.randn(B, H, cap, D, device=cuda).to(torch.bfloat16) for _ in range(L)]
    pk = [torch.randn(H, int(cu_q[-1]), D, device=cuda).to(torch.bfloat16) for _ in range(L)]
    pv = [torch.randn(H, int(cu_q[-1]), D, device=cuda).to(torch.bfloat16) for _ in range(L)]
    host = lambda ts: [t.float().cpu().numpy() for t in ts]
    acc = w.accepted.cpu().tolist()
    keep = [row[:a] for row, a in zip(w.keep.cpu().tolist(), acc)]
    rk, rv, _ = okv.append_store(host(bufk), host(bufv), sl.cpu().tolist(), cu_q.tolist(), keep, acc,
                                 list(range(B)), host(pk), host(pv))
    cast_b200.append_store_inplace(bufk, bufv, sl, cu_t[:-1], w.keep, w.accepted, pk, pv)
    assert _lib.device_error() == 0
    for li in range(L):
        assert np.array_equal(bufk[li].float().cpu().numpy(), rk[li])
        assert np.array_equal(bufv[li].float().cpu().numpy(), rv[li])


# ---------------------------------------------------------------------- gather cache
def test_gather_cache_matches_reference_golden(cuda, golden):
    g = golden("gather.npz")
    to = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    cache = types.SimpleNamespace(key_cache=[to(x) for x in g["in_k"]], value_cache=[to(x) for x in g["in_v"]],
                                  _seen_tokens=0)
    cast_b200.gather_cache(cache, int(g["n_prefix"]), g["keep"].tolist())
    assert _lib.device_error() == 0
    assert np.array_equal(torch.stack(cache.key_cache).cpu().numpy(), g["out_k"])
    assert np.array_equal(torch.stack(cache.value_cache).cpu().numpy(), g["out_v"])
    assert cache._seen_tokens == int(g["n_prefix"]) + len(g["keep"])


def test_gather_cache_layers_layout_bf16(cuda):
    # the newer cache layout (layers[i].keys / .values), several batch rows, empty keep
    L, B, H, S, D = 3, 2, 8, 200, 128
    layers = [types.SimpleNamespace(keys=torch.randn(B, H, S, D, device=cuda).to(torch.bfloat16),
                                    values=torch.randn(B, H, S, D, device=cuda).to(torch.bfloat16))
              for _ in range(L)]
    ks = [x.keys.float().cpu().numpy() for x in layers]
    vs = [x.values.float().cpu().numpy() for x in layers]
    for n_prefix, keep in ((150, [0, 3, 7, 49]), (180, [])):
        cache = types.SimpleNamespace(layers=[types.SimpleNamespace(keys=x.keys, values=x.values) for x in layers])
        rk, rv = okv.gather_cache(ks, vs, n_prefix, keep)
        cast_b200.gather_cache(cache, n_prefix, keep)
        assert _lib.device_error() == 0
        for li in range(L):
            assert np.array_equal(cache.layers[li].keys.float().cpu().numpy(), rk[li])
            assert np.array_equal(cache.layers[li].values.float().cpu().numpy(), rv[li])
