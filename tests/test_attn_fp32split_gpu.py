"""fp32 tree attention through the tensor cores (CAST_F32_SPLIT), against the CPU oracle.

The reference hook hands the kernel fp32 copies (cast_trees/serving.py:68-71) and the
path's bound for fp32 inputs is 1e-4 max abs. The split path carries q, k, v and the
probabilities as bf16 hi + lo pairs (three-term products) and skips the MMAs of lo
parts that are all zero; these tests run general fp32 data (every lo part non-zero),
fp32 copies of bf16 data (every lo part zero), mixed cases, configuration 3 itself,
the tensor-core kernel's ragged edge shapes, and compare with the exact CUDA-core path.
"""
import numpy as np
import pytest
import torch

import cast_b200
from cast_b200 import _lib, workloads
from oracle import attn as oattn
from oracle import tree as otree

pytestmark = pytest.mark.gpu

TOL = 1e-4


def _scenario(S_list, P_list, Hq=32, Hkv=8, seed=5, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    rng = np.random.default_rng(seed)
    parents = []
    for P in P_list:
        parents += [-1] + [int(rng.integers(0, i)) for i in range(1, P)]
    cu_q = np.concatenate([[0], np.cumsum(P_list)]).astype(np.int32)
    cu_kv = np.concatenate([[0], np.cumsum(np.array(S_list) + np.array(P_list))]).astype(np.int32)
    mk = lambda n, h: torch.randn(n, h, 128, generator=g) * scale
    return dict(q=mk(int(cu_q[-1]), Hq), k=mk(int(cu_kv[-1]), Hkv), v=mk(int(cu_kv[-1]), Hkv), cu_q=cu_q,
                cu_kv=cu_kv, prefix=np.array(S_list, np.int32), pack=np.array(P_list, np.int32),
                parent=np.array(parents, np.int32))


def _words(sc):
    cu = sc["cu_q"]
    return [otree.ancestor_words(sc["parent"][cu[b]:cu[b + 1]]) for b in range(len(cu) - 1)]


def _run(sc, dev, q=None, k=None, v=None, path="split"):
    q = sc["q"] if q is None else q
    k = sc["k"] if k is None else k
    v = sc["v"] if v is None else v
    t = lambda a: torch.as_tensor(a).to(dev)
    out = cast_b200.varlen_tree_attention(q.to(dev), k.to(dev), v.to(dev), t(sc["cu_q"]), t(sc["cu_kv"]),
                                          t(sc["prefix"]), t(sc["pack"]), None, parent=t(sc["parent"]),
                                          fp32_path=path)
    assert _lib.device_error() == 0
    return out.cpu()


def _oracle(sc, q=None, k=None, v=None):
    q = sc["q"] if q is None else q
    k = sc["k"] if k is None else k
    v = sc["v"] if v is None else v
    return oattn.tree_attention(q, k, v, sc["cu_q"], sc["cu_kv"], sc["prefix"], sc["pack"], _words(sc))


def test_plan_is_the_split_tensor_core_path(cuda):
    q = torch.zeros(130, 32, 128, device=cuda)
    k = torch.zeros(1000, 8, 128, device=cuda)
    assert cast_b200.attention_plan(q, k, k, q, 1, 130, 1000)[0] == "tcgen05_split"
    assert cast_b200.attention_plan(q, k, k, q, 1, 130, 1000, fp32_path="exact")[0] == "simt"


@pytest.mark.parametrize("lo", ["all", "none", "k_only", "q_v_only"])
def test_low_parts_present_or_absent(cuda, lo):
    sc = _scenario([300, 0, 1100, 77, 4000], [128, 257, 17, 64, 1], seed=11)
    bf = lambda x: x.to(torch.bfloat16).float()
    q, k, v = sc["q"], sc["k"], sc["v"]
    if lo == "none":
        q, k, v = bf(q), bf(k), bf(v)        # fp32 copies of bf16 data, as the reference hook makes
    elif lo == "k_only":
        q, v = bf(q), bf(v)
    elif lo == "q_v_only":
        k = bf(k)
    err = (_run(sc, cuda, q, k, v) - _oracle(sc, q, k, v)).abs().max().item()
    assert err < TOL, err


@pytest.mark.parametrize("Hq,Hkv", [(32, 8), (8, 8), (16, 8), (64, 4)])
def test_ragged_edge_shapes(cuda, Hq, Hkv):
    # a pure pack (S = 0), a one-token pack, prefixes ending inside a key tile, packs wider than 64
    sc = _scenario([0, 1, 127, 129, 700, 64, 2000], [70, 1, 33, 128, 300, 129, 17], Hq=Hq, Hkv=Hkv, seed=21)
    err = (_run(sc, cuda) - _oracle(sc)).abs().max().item()
    assert err < TOL, err


@pytest.mark.parametrize("scale", [1.0, 2.0])
def test_key_splits_and_input_scale(cuda, scale):
    # two long prefixes (the launch splits the keys, partials are merged). hi + lo carries ~16 bits,
    # so the logits' absolute error grows with |q| |k| and the output's with |v|: the 1e-4 bound is
    # the unit-scale one, and at twice the scale (logits 4x, values 2x) the bound is scaled the same way
    sc = _scenario([30000, 17001], [9, 130], seed=6, scale=scale)
    q = sc["q"].to(cuda)
    kernel, n_split, _ = cast_b200.attention_plan(q, sc["k"].to(cuda), sc["v"].to(cuda), q, 2, 130, 30009)
    assert kernel == "tcgen05_split" and n_split > 1
    err = (_run(sc, cuda) - _oracle(sc)).abs().max().item()
    assert err < TOL * scale ** 3, err


def test_split_and_exact_paths_agree(cuda):
    sc = _scenario([1000, 37, 4096, 5], [128, 64, 100, 1], seed=22)
    a = _run(sc, cuda, path="split")
    b = _run(sc, cuda, path="exact")
    assert (a - b).abs().max().item() < TOL


def test_configuration_3_in_fp32(cuda):
    # the bench's workload with fp32 inputs: GPU-built trees, q/k/v N(0,1) * 0.5 drawn in fp32
    w = workloads.config(3, torch.float32)
    lay = w.layout()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    idx, lp = cast_b200.block_topk_device(t(w.logits_batch()), 8)
    cu_q = t(lay["cu_q"])
    trees = cast_b200.build_trees(idx, lp, 127, 8, max_budget=127, cu_q=cu_q, total_q=lay["total_q"])
    q, k, v = w.make_qkv(cuda)
    assert q.dtype == torch.float32
    out = torch.empty_like(q)
    assert cast_b200.attention_plan(q, k, v, out, w.B, lay["max_pack"], lay["max_kv"])[0] == "tcgen05_split"
    cast_b200.varlen_tree_attention(q, k, v, cu_q, t(lay["cu_kv"]), t(lay["prefix_len"]), t(lay["pack_len"]), None,
                                    parent=trees.pack_parent, max_pack=lay["max_pack"], max_kv=lay["max_kv"], out=out)
    assert _lib.device_error() == 0
    pp = trees.pack_parent.cpu().numpy()
    cq, ckv = lay["cu_q"], lay["cu_kv"]
    for b in np.random.default_rng(33).choice(w.B, size=6, replace=False).tolist():
        S, P = w.S[b], w.P[b]
        ref = oattn.tree_attention(q[cq[b]:cq[b + 1]].cpu(), k[ckv[b]:ckv[b + 1]].cpu(), v[ckv[b]:ckv[b + 1]].cpu(),
                                   [0, P], [0, S + P], [S], [P], [otree.ancestor_words(pp[cq[b]:cq[b + 1]])])
        err = (out[cq[b]:cq[b + 1]].cpu() - ref).abs().max().item()
        assert err < TOL, (b, err)
