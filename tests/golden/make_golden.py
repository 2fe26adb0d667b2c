"""Regenerate the golden vectors by running the reference package itself.

    python tests/golden/make_golden.py --reference <path to the CAST checkout>

The reference (js-lee-AI/CAST, package ``cast_trees``) is imported from the
given checkout; its decoder modules need ``dflash``, which is replaced by an
inert stub module since only ``walk_tree`` is called. Every output below is
what the reference computed; the CPU tests pin the oracle against them and the
GPU tests pin the CUDA library against them.

Files written next to this script:
  tree_cfg1.npz     block_topk of rng(0).normal(scale=5, (15, 64)) and
                    build_tree at N = 16 and N = 127 (configuration 1 and the
                    quickstart's expected accepted length)
  tree_cases.npz    build_tree on assorted (L, V, k, budget) cases, including
                    integer logits that force ties in both the sort and the heap
  topk_vocab.npz    block_topk on full-vocabulary rows (V = 151936, 128256)
  attn_cfg1.npz     config 1 attention through the reference's dense mask
                    (verify.tree_attention_mask + SDPA), fp32
  attn_ragged.npz   a seeded ragged scenario built like tests/test_tree_attn.py,
                    scored by that file's reference(), at a reduced head count
  walk.npz          decode.walk_tree greedy paths on seeded logits
  select.npz        tree.select_global_topk on seeded forests (several totals,
                    and a forest whose scores tie across trees)
  append.npz        serving.BatchedServer._append_store on small seeded stores:
                    append in place, compaction (a request leaves), growth
  gather.npz        verify.gather_cache on a small seeded two-layer cache
"""
import argparse
import importlib
import math
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _import_reference(path):
    sys.path.insert(0, str(path))
    stub = types.ModuleType("dflash")
    stub_model = types.ModuleType("dflash.model")
    stub_model.extract_context_feature = lambda *a, **k: None
    stub.model = stub_model
    sys.modules.setdefault("dflash", stub)
    sys.modules.setdefault("dflash.model", stub_model)
    tree = importlib.import_module("cast_trees.tree")
    verify = importlib.import_module("cast_trees.verify")
    decode = importlib.import_module("cast_trees.decode")
    spec = importlib.util.spec_from_file_location("ref_test_tree_attn",
                                                  Path(path) / "tests" / "test_tree_attn.py")
    tta = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(tta)
    return tree, verify, decode, tta


def _nodes_arrays(nodes):
    return dict(token=np.array([n.token for n in nodes], dtype=np.int64),
                depth=np.array([n.depth for n in nodes], dtype=np.int64),
                parent=np.array([n.parent for n in nodes], dtype=np.int64),
                score=np.array([n.score for n in nodes], dtype=np.float64))


def tree_cfg1(tree):
    logits = np.random.default_rng(0).normal(scale=5, size=(15, 64))
    idx, lp = tree.block_topk(logits)
    out = dict(idx=idx, lp=lp)
    for n in (16, 127):
        nodes = tree.build_tree(idx, lp, n)
        for key, val in _nodes_arrays(nodes).items():
            out[f"n{n}_{key}"] = val
        out[f"n{n}_expected_len"] = np.float64(tree.expected_accepted_length(nodes))
    np.savez_compressed(HERE / "tree_cfg1.npz", **out)


# (name, seed, L, V, k, budget, scale, integer) - the integer cases round the
# logits so equal log-probs, equal path scores and equal depths all occur.
TREE_CASES = [
    ("rand63", 0, 15, 100, 8, 63, 3.0, False),
    ("rand127", 1, 15, 200, 8, 127, 3.0, False),
    ("rand256", 2, 15, 500, 8, 256, 5.0, False),
    ("small3", 3, 3, 100, 4, 20, 3.0, False),
    ("k4_300", 4, 6, 50, 4, 300, 2.0, False),
    ("exhaust", 5, 3, 10, 3, 100, 1.0, False),     # universe of 39 nodes < budget
    ("ties_int", 6, 15, 40, 8, 127, 1.0, True),
    ("ties_flat", 7, 8, 16, 8, 200, 0.0, True),    # all logits equal
    ("ties_k2", 8, 10, 12, 2, 150, 0.6, True),
    ("budget0", 9, 15, 64, 8, 0, 5.0, False),
    ("k1_chain", 10, 15, 64, 1, 20, 5.0, False),
]


def tree_cases(tree):
    out = {}
    for name, seed, L, V, k, budget, scale, integer in TREE_CASES:
        x = np.random.default_rng(seed).normal(scale=max(scale, 1e-9), size=(L, V))
        if integer:
            x = np.round(x)
        if scale == 0.0:
            x = np.zeros((L, V))
        idx, lp = tree.block_topk(x, max(k, 1))
        nodes = tree.build_tree(idx, lp, budget, k)
        out[f"{name}_logits"] = x
        out[f"{name}_idx"] = idx
        out[f"{name}_lp"] = lp
        for key, val in _nodes_arrays(nodes).items():
            out[f"{name}_{key}"] = val
    out["names"] = np.array([c[0] for c in TREE_CASES])
    out["params"] = np.array([[c[1], c[2], c[3], c[4], c[5]] for c in TREE_CASES], dtype=np.int64)
    np.savez_compressed(HERE / "tree_cases.npz", **out)


# full-vocabulary rows: logits are regenerated from the seed in the tests
VOCAB_CASES = [("v151936", (1, 0), 151936), ("v128256", (2, 0), 128256)]


def topk_vocab(tree):
    out = {}
    for name, seed, V in VOCAB_CASES:
        x = np.random.default_rng(list(seed)).normal(scale=5, size=(15, V))
        idx, lp = tree.block_topk(x)
        out[f"{name}_idx"] = idx
        out[f"{name}_lp"] = lp
        nodes = tree.build_tree(idx, lp, 127)
        for key, val in _nodes_arrays(nodes).items():
            out[f"{name}_n127_{key}"] = val
        out[f"{name}_seed"] = np.array(seed, dtype=np.int64)
    np.savez_compressed(HERE / "topk_vocab.npz", **out)


def attn_cfg1(tree, verify):
    logits = np.random.default_rng(0).normal(scale=5, size=(15, 64))
    idx, lp = tree.block_topk(logits)
    nodes = tree.build_tree(idx, lp, 16)
    S, P, Hq, Hkv, D = 512, 17, 32, 8, 128
    g = torch.Generator().manual_seed(0)
    q = torch.randn(P, Hq, D, generator=g)
    k = torch.randn(S + P, Hkv, D, generator=g)
    v = torch.randn(S + P, Hkv, D, generator=g)
    mask = verify.tree_attention_mask(S, nodes, "cpu", torch.float32)
    o = torch.nn.functional.scaled_dot_product_attention(
        q.transpose(0, 1)[None], k.transpose(0, 1)[None], v.transpose(0, 1)[None],
        attn_mask=mask, scale=1.0 / math.sqrt(D), enable_gqa=True)
    np.savez_compressed(HERE / "attn_cfg1.npz", out=o[0].transpose(0, 1).contiguous().numpy(),
                        parent=np.array([n.parent for n in nodes], dtype=np.int64),
                        S=S, P=P)


def ragged_scenario(seed=11, B=6, Hq=8, Hkv=2, D=64, s_range=(0, 300), p_range=(1, 64)):
    """Seeded ragged batch built like tests/test_tree_attn.py:11-37, on the CPU.

    Draw order per request: prefix length, pack length, parents, then q, k, v.
    With the defaults, prefix lengths may be 0 and packs may hold a single
    token (edge cases); s_range=(200, 400), p_range=(2, 64) with B=8, Hq=32,
    Hkv=8, D=128 is the reference test's own scenario.
    """
    g = torch.Generator().manual_seed(seed)
    qs, ks, vs, bits, reqs = [], [], [], [], []
    cu_q, cu_kv = [0], [0]
    for _ in range(B):
        S = int(torch.randint(s_range[0], s_range[1], (1,), generator=g))
        P = int(torch.randint(p_range[0], p_range[1], (1,), generator=g))
        parent = [-1] + [int(torch.randint(0, i, (1,), generator=g)) for i in range(1, P)]
        qs.append(torch.randn(P, Hq, D, generator=g))
        ks.append(torch.randn(S + P, Hkv, D, generator=g))
        vs.append(torch.randn(S + P, Hkv, D, generator=g))
        for i in range(P):
            w, j = 0, i
            while j != -1:
                w |= 1 << j
                j = parent[j]
            bits.append(w)
        cu_q.append(cu_q[-1] + P)
        cu_kv.append(cu_kv[-1] + S + P)
        reqs.append((S, P, parent))
    parents = np.full(cu_q[-1], -1, dtype=np.int32)
    for b, (S, P, parent) in enumerate(reqs):
        parents[cu_q[b]:cu_q[b] + P] = parent
    return dict(q=torch.cat(qs), k=torch.cat(ks), v=torch.cat(vs),
                cu_q=torch.tensor(cu_q, dtype=torch.int32), cu_kv=torch.tensor(cu_kv, dtype=torch.int32),
                prefix=np.array([r[0] for r in reqs], np.int32),
                pack=np.array([r[1] for r in reqs], np.int32),
                bits=np.array(bits, dtype=np.uint64).view(np.int64), parent=parents, reqs=reqs)


def attn_ragged(tta):
    scen = ragged_scenario()
    ref = tta.reference(scen)
    np.savez_compressed(HERE / "attn_ragged.npz", out=ref.numpy(), seed=11)


def walk(tree, decode):
    out = {}
    rng = np.random.default_rng(21)
    for c in range(6):
        idx, lp = tree.block_topk(rng.normal(scale=3, size=(15, 12)), 4)
        nodes = tree.build_tree(idx, lp, 40, 4)
        # logits that follow the tree for a few levels, then diverge
        P = 1 + len(nodes)
        logits = rng.normal(size=(P, 12))
        for i in range(-1, len(nodes)):
            kids = [j for j, n in enumerate(nodes) if n.parent == i]
            if kids and rng.random() < 0.8:
                logits[i + 1, nodes[kids[int(rng.integers(len(kids)))]].token] += 10.0
        path, bonus = decode.walk_tree(nodes, torch.tensor(logits), 0.0)
        out[f"c{c}_parent"] = np.array([n.parent for n in nodes], dtype=np.int64)
        out[f"c{c}_token"] = np.array([n.token for n in nodes], dtype=np.int64)
        out[f"c{c}_logits"] = logits
        out[f"c{c}_path"] = np.array(path, dtype=np.int64)
        out[f"c{c}_bonus"] = np.int64(bonus)
    np.savez_compressed(HERE / "walk.npz", **out)


def _forest_arrays(trees, prefix, out):
    mb = max(1, max(len(t) for t in trees))
    B = len(trees)
    tok = np.zeros((B, mb), np.int64)
    dep = np.zeros((B, mb), np.int64)
    par = np.full((B, mb), -1, np.int64)
    sc = np.zeros((B, mb), np.float64)
    for b, nodes in enumerate(trees):
        for j, nd in enumerate(nodes):
            tok[b, j], dep[b, j], par[b, j], sc[b, j] = nd.token, nd.depth, nd.parent, nd.score
    out[prefix + "token"], out[prefix + "depth"], out[prefix + "parent"], out[prefix + "score"] = tok, dep, par, sc
    out[prefix + "count"] = np.array([len(t) for t in trees], np.int64)


SELECT_TOTALS = (0, 1, 17, 64, 200, 10000, -5)


def select(tree):
    out = {}
    rng = np.random.default_rng(31)
    # seeded forests of unequal trees (the reference test's shape: 8 trees, budget 48)
    forests = {"rand": [tree.build_tree(*tree.block_topk(rng.normal(scale=3, size=(15, 40))), budget=48)
                        for _ in range(8)],
               "ties": [tree.build_tree(*tree.block_topk(np.round(rng.normal(scale=2, size=(6, 5)))), budget=12)
                        for _ in range(5)]}
    # identical trees: every score ties across trees, so (tree, node) order decides
    same = tree.build_tree(*tree.block_topk(rng.normal(scale=3, size=(8, 20))), budget=20)
    forests["same"] = [same, same, same]
    for name, trees in forests.items():
        _forest_arrays(trees, f"{name}_in_", out)
        for total in SELECT_TOTALS:
            _forest_arrays(tree.select_global_topk(trees, total), f"{name}_t{total}_", out)
    out["totals"] = np.array(SELECT_TOTALS, np.int64)
    np.savez_compressed(HERE / "select.npz", **out)


def append(serving):
    """_append_store with a stand-in `self` (only .device is read) and PACK_KV set per case."""
    out = {}
    rng = np.random.default_rng(41)
    g = torch.Generator().manual_seed(41)
    L, H, D = 2, 2, 16
    cases = {"inplace": dict(B=3, cap=12, store_len=[3, 5, 0], rows=[0, 1, 2]),
             "compact": dict(B=4, cap=12, store_len=[4, 2, 6, 1], rows=[0, 2, 3]),
             "grow": dict(B=3, cap=8, store_len=[6, 2, 7], rows=[1, 2])}
    for name, c in cases.items():
        B, cap, sl, rows = c["B"], c["cap"], c["store_len"], c["rows"]
        buf_k = [torch.zeros((B, H, cap, D)) for _ in range(L)]
        buf_v = [torch.zeros((B, H, cap, D)) for _ in range(L)]
        for li in range(L):
            for b in range(B):
                buf_k[li][b, :, :sl[b]] = torch.randn(H, sl[b], D, generator=g)
                buf_v[li][b, :, :sl[b]] = torch.randn(H, sl[b], D, generator=g)
        pack = [int(rng.integers(3, 7)) for _ in range(B)]
        cu_q = [0]
        for p in pack:
            cu_q.append(cu_q[-1] + p)
        keep, accepted = [], []
        for b in range(B):
            path = sorted(rng.choice(np.arange(1, pack[b]), size=int(rng.integers(0, pack[b])), replace=False))
            keep.append([0] + [int(x) for x in path])
            accepted.append(len(path) + 1)
        pk = [torch.randn(H, cu_q[-1], D, generator=g) for _ in range(L)]
        pv = [torch.randn(H, cu_q[-1], D, generator=g) for _ in range(L)]
        serving.PACK_KV["k"], serving.PACK_KV["v"] = pk, pv
        me = types.SimpleNamespace(device=torch.device("cpu"))
        ins_k = [x.clone() for x in buf_k]
        ins_v = [x.clone() for x in buf_v]
        nk, nv, new_len = serving.BatchedServer._append_store(me, buf_k, buf_v, sl, cu_q, keep, accepted, rows)
        out[f"{name}_in_k"] = torch.stack(ins_k).numpy()
        out[f"{name}_in_v"] = torch.stack(ins_v).numpy()
        out[f"{name}_pack_k"] = torch.stack(pk).numpy()
        out[f"{name}_pack_v"] = torch.stack(pv).numpy()
        out[f"{name}_store_len"] = np.array(sl, np.int64)
        out[f"{name}_cu_q"] = np.array(cu_q, np.int64)
        out[f"{name}_rows"] = np.array(rows, np.int64)
        out[f"{name}_accepted"] = np.array(accepted, np.int64)
        kk = np.full((B, max(len(k) for k in keep)), -1, np.int64)
        for b in range(B):
            kk[b, :len(keep[b])] = keep[b]
        out[f"{name}_keep"] = kk
        out[f"{name}_out_k"] = torch.stack(nk).numpy()
        out[f"{name}_out_v"] = torch.stack(nv).numpy()
        out[f"{name}_new_len"] = np.array(new_len, np.int64)
    np.savez_compressed(HERE / "append.npz", **out)


def gather(verify):
    g = torch.Generator().manual_seed(51)
    L, B, H, S, D = 2, 1, 2, 20, 16
    cache = types.SimpleNamespace(key_cache=[torch.randn(B, H, S, D, generator=g) for _ in range(L)],
                                  value_cache=[torch.randn(B, H, S, D, generator=g) for _ in range(L)])
    in_k = torch.stack(cache.key_cache).numpy().copy()
    in_v = torch.stack(cache.value_cache).numpy().copy()
    n_prefix, keep = 12, [0, 2, 3, 6]
    verify.gather_cache(cache, n_prefix, keep)
    np.savez_compressed(HERE / "gather.npz", in_k=in_k, in_v=in_v, n_prefix=np.int64(n_prefix),
                        keep=np.array(keep, np.int64), out_k=torch.stack(cache.key_cache).numpy(),
                        out_v=torch.stack(cache.value_cache).numpy())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path to the CAST checkout")
    ap.add_argument("--only", default="", help="comma-separated subset of the files to write (by stem)")
    args = ap.parse_args()
    tree, verify, decode, tta = _import_reference(args.reference)
    want = set(x for x in args.only.split(",") if x)
    run = lambda stem: not want or stem in want
    if run("tree_cfg1"):
        tree_cfg1(tree)
    if run("tree_cases"):
        tree_cases(tree)
    if run("topk_vocab"):
        topk_vocab(tree)
    if run("attn_cfg1"):
        attn_cfg1(tree, verify)
    if run("attn_ragged"):
        attn_ragged(tta)
    if run("walk"):
        walk(tree, decode)
    if run("select"):
        select(tree)
    if run("append"):
        append(importlib.import_module("cast_trees.serving"))
    if run("gather"):
        gather(verify)
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
