"""Greedy accept lengths through the GPU path equal the reference's.

A verify round (cast_trees/serving.py:292-351): trees from the drafter's block
scores, one ancestor-masked attention pass, target logits per packed row, then
the greedy tree walk of cast_trees/decode.py:96-103. No target model exists
here, so the target head is synthetic and fixed: each packed row's logits are a
seeded projection of its attention output (all query heads) plus the
drafter's scores for the next position, scaled so that the attention term
decides a good share of the argmaxes. The walk is run on logits from the CUDA
path (GPU trees + GPU attention) and from the oracle path (numpy trees + fp32
attention); the accepted paths and bonus tokens must be identical.
"""
import numpy as np
import pytest
import torch

import cast_b200
from cast_b200 import _lib
from oracle import attn as oattn
from oracle import tree as otree

pytestmark = pytest.mark.gpu

V_SMALL = 64     # drafter vocabulary of the synthetic round
L_BLOCK = 15


def _round(dev, dtype, seed, B=8, n_nodes=31, Hq=32, Hkv=8, D=128):
    rng = np.random.default_rng(seed)
    block = [rng.normal(scale=3.0, size=(L_BLOCK, V_SMALL)) for _ in range(B)]
    S = [int(rng.integers(64, 600)) for _ in range(B)]
    P = [n_nodes + 1] * B
    cu_q = np.concatenate([[0], np.cumsum(P)]).astype(np.int32)
    cu_kv = np.concatenate([[0], np.cumsum(np.array(S) + np.array(P))]).astype(np.int32)
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(int(cu_q[-1]), Hq, D, generator=g)
    k = torch.randn(int(cu_kv[-1]), Hkv, D, generator=g)
    v = torch.randn(int(cu_kv[-1]), Hkv, D, generator=g)
    W = torch.randn(Hq * D, V_SMALL, generator=g, dtype=torch.float64) / np.sqrt(Hq * D)
    return dict(block=block, S=S, P=P, cu_q=cu_q, cu_kv=cu_kv, q=q, k=k, v=v, W=W, B=B, n=n_nodes)


def _target_logits(o, W, block, depth, scale):
    """[P, V] logits of one pack: projection of the attention output + drafter scores of the next position."""
    proj = o.reshape(o.shape[0], -1).double() @ W            # [P, V]
    nxt = np.zeros((o.shape[0], V_SMALL))
    for r, d in enumerate(depth):                             # row r predicts position d + 1
        if d < L_BLOCK:
            nxt[r] = block[d]
    return scale * proj.numpy() + nxt


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("seed", [0, 1])
def test_greedy_accept_lengths_identical(cuda, dtype, seed):
    rd = _round(cuda, dtype, seed)
    B, n = rd["B"], rd["n"]
    # CUDA path: trees and attention on the GPU
    logits_d = torch.from_numpy(np.stack(rd["block"])).to(cuda)
    idx, lp = cast_b200.block_topk_device(logits_d, 8)
    trees = cast_b200.build_trees(idx, lp, n, 8, cu_q=torch.from_numpy(rd["cu_q"]).to(cuda),
                                  total_q=int(rd["cu_q"][-1]))
    t = lambda a: torch.from_numpy(np.asarray(a, dtype=np.int32)).to(cuda)
    out = cast_b200.varlen_tree_attention(rd["q"].to(cuda, dtype), rd["k"].to(cuda, dtype), rd["v"].to(cuda, dtype),
                                          t(rd["cu_q"]), t(rd["cu_kv"]), t(rd["S"]), t(rd["P"]), None,
                                          parent=trees.pack_parent)
    assert _lib.device_error() == 0
    out = out.float().cpu()
    # oracle path: numpy trees, fp32 attention on the same (rounded) inputs
    otrees = [otree.build_tree(*otree.block_topk(rd["block"][b]), n) for b in range(B)]
    words = [otree.ancestor_words(otree.pack_parent(tr.parent)) for tr in otrees]
    q32, k32, v32 = (rd[x].to(dtype).float() for x in ("q", "k", "v"))
    ref = oattn.tree_attention(q32, k32, v32, rd["cu_q"], rd["cu_kv"], rd["S"], rd["P"], words)
    # the synthetic head's scale: attention term comparable to the drafter's score gaps
    scale = 3.0 / float((ref.reshape(ref.shape[0], -1).double() @ rd["W"]).std())
    lengths = []
    for b in range(B):
        q0, q1 = int(rd["cu_q"][b]), int(rd["cu_q"][b + 1])
        tr = otrees[b]
        assert np.array_equal(trees.parent[b, :n].cpu().numpy(), tr.parent)
        assert np.array_equal(trees.token[b, :n].cpu().numpy(), tr.token)
        depth = [0] + tr.depth.tolist()
        z_gpu = _target_logits(out[q0:q1], rd["W"], rd["block"][b], depth, scale)
        z_ref = _target_logits(ref[q0:q1], rd["W"], rd["block"][b], depth, scale)
        path_gpu, bonus_gpu = otree.walk_tree_greedy(tr.parent, tr.token, z_gpu)
        path_ref, bonus_ref = otree.walk_tree_greedy(tr.parent, tr.token, z_ref)
        assert path_gpu == path_ref and bonus_gpu == bonus_ref, (b, path_gpu, path_ref)
        lengths.append(len(path_ref) + 1)
    # the walk is not trivial: some rounds accept several tokens, not every round accepts all
    assert max(lengths) >= 3 and min(lengths) <= n
