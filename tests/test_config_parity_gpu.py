"""Attention parity on the benchmark configurations themselves (GPU, through the C ABI).

Each case builds the whole configuration the way the bench does: fp64 block
scores of every sequence on the device, GPU block_topk + build_tree writing
the pack parents, q/k/v from the configuration's recipe (N(0,1) * 0.5, bf16),
and one call of the public attention API with host bounds (the launch plan
the bench times: tensor-core kernel, same key splits). A seeded subset of the
sequences is then recomputed by the CPU oracle from the same inputs and the
GPU's tree; the bound is the path's bf16 tolerance, 2e-2 max abs.
"""
import numpy as np
import pytest
import torch

import cast_b200
from cast_b200 import _lib, workloads
from oracle import attn as oattn
from oracle import tree as otree

pytestmark = pytest.mark.gpu

TOL_BF16 = 2e-2


def _device_round(w, dev):
    lay = w.layout()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    logits = t(w.logits_batch())
    idx, lp = cast_b200.block_topk_device(logits, 8)
    del logits
    cu_q = t(lay["cu_q"])
    budget = torch.tensor(w.N, dtype=torch.int32, device=dev)
    trees = cast_b200.build_trees(idx, lp, budget, 8, max_budget=max(w.N), cu_q=cu_q, total_q=lay["total_q"])
    q, k, v = w.make_qkv(dev)
    out = torch.empty_like(q)
    plan = cast_b200.attention_plan(q, k, v, out, w.B, lay["max_pack"], lay["max_kv"])
    cast_b200.varlen_tree_attention(q, k, v, cu_q, t(lay["cu_kv"]), t(lay["prefix_len"]), t(lay["pack_len"]),
                                    None, parent=trees.pack_parent, max_pack=lay["max_pack"],
                                    max_kv=lay["max_kv"], out=out)
    assert _lib.device_error() == 0
    return lay, idx, lp, trees, (q, k, v), out, plan


def _oracle_subset(lay, trees, qkv, ids):
    """Oracle output of sequences `ids` (rows in pack order, concatenated)."""
    q, k, v = qkv
    cq, ckv = lay["cu_q"], lay["cu_kv"]
    qs, ks, vs, words, cu_q, cu_kv = [], [], [], [], [0], [0]
    pp = trees.pack_parent.cpu().numpy()
    for b in ids:
        qs.append(q[cq[b]:cq[b + 1]].float().cpu())
        ks.append(k[ckv[b]:ckv[b + 1]].float().cpu())
        vs.append(v[ckv[b]:ckv[b + 1]].float().cpu())
        words.append(otree.ancestor_words(pp[cq[b]:cq[b + 1]]))
        cu_q.append(cu_q[-1] + int(cq[b + 1] - cq[b]))
        cu_kv.append(cu_kv[-1] + int(ckv[b + 1] - ckv[b]))
    S = [int(lay["prefix_len"][b]) for b in ids]
    P = [int(lay["pack_len"][b]) for b in ids]
    return oattn.tree_attention(torch.cat(qs), torch.cat(ks), torch.cat(vs), cu_q, cu_kv, S, P, words)


@pytest.mark.parametrize("cfg, n_check, n_tree", [(2, 16, 2), (3, 16, 2), (4, 8, 1)])
def test_configuration_attention_matches_oracle(cuda, cfg, n_check, n_tree):
    w = workloads.config(cfg)
    lay, idx, lp, trees, qkv, out, plan = _device_round(w, cuda)
    kernel, n_split, _ = plan
    assert kernel == "tcgen05"
    if cfg == 4:
        assert n_split > 1          # 64 (sequence, head) pairs: the launch splits the keys
    ids = sorted(np.random.default_rng(100 + cfg).choice(w.B, size=n_check, replace=False).tolist())
    # the trees the attention used are the reference algorithm's trees
    for b in ids[:n_tree]:
        oi, ol = otree.block_topk(w.logits(b))
        ref = otree.build_tree(oi, ol, w.N[b])
        q0, q1 = lay["cu_q"][b], lay["cu_q"][b + 1]
        assert trees.pack_parent[q0:q1].cpu().tolist() == otree.pack_parent(ref.parent).tolist()
    expect = _oracle_subset(lay, trees, qkv, ids)
    got = torch.cat([out[lay["cu_q"][b]:lay["cu_q"][b + 1]].float().cpu() for b in ids])
    err = (got - expect).abs()
    assert err.max().item() < TOL_BF16, (cfg, err.max().item())
    assert err.mean().item() < 5e-3, (cfg, err.mean().item())
