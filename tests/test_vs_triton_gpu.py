"""This library's attention and the reference's own Triton kernel on the same inputs (GPU).

The reference kernel (cast_trees/tree_attn.py:17-139) is imported unmodified from
the reference package installed beside the repo (baseline/_ref); without it the
test is skipped. It takes packs of at most 64 tokens, so the cases are
configuration 1 and the configuration-2 sequences with N <= 63. Both outputs
must be within the path's tolerance of the CPU oracle (fp32 1e-4 for ours; the
reference's fp32 runs its dots in tf32, so it gets the reference test's own
5e-2 bound), and within 2e-2 of each other for bf16.
"""
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

import cast_b200
from cast_b200 import _lib, workloads
from cast_b200.bench_case import _ancestor_bits
from oracle import attn as oattn
from oracle import tree as otree

pytestmark = pytest.mark.gpu

REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


def _ref_module():
    if not (REF / "cast_trees" / "tree_attn.py").exists():
        pytest.skip("reference package not installed in baseline/_ref")
    sys.path.insert(0, str(REF))
    try:
        from cast_trees import tree_attn
    finally:
        sys.path.remove(str(REF))
    return tree_attn


@pytest.mark.parametrize("cfg, dtype", [(1, torch.float32), (1, torch.bfloat16), (2, torch.bfloat16)])
def test_ours_and_reference_kernel_against_oracle(cuda, cfg, dtype):
    ref_ta = _ref_module()
    w = workloads.config(cfg, dtype)
    if cfg == 2:
        w = w.shard([b for b in range(w.B) if w.N[b] <= 63])
    lay = w.layout()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    idx, lp = cast_b200.block_topk_device(t(w.logits_batch()), 8)
    cu_q, cu_kv, prefix, pack = t(lay["cu_q"]), t(lay["cu_kv"]), t(lay["prefix_len"]), t(lay["pack_len"])
    trees = cast_b200.build_trees(idx, lp, torch.tensor(w.N, dtype=torch.int32, device=cuda), 8,
                                  max_budget=max(w.N), cu_q=cu_q, total_q=lay["total_q"])
    bits = _ancestor_bits(trees.pack_parent, cu_q, pack, 15)
    q, k, v = w.make_qkv(cuda, dtype)
    ours = cast_b200.varlen_tree_attention(q, k, v, cu_q, cu_kv, prefix, pack, None, parent=trees.pack_parent)
    theirs = ref_ta.varlen_tree_attention(q, k, v, cu_q, cu_kv, prefix, pack, bits)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    pp = trees.pack_parent.cpu().numpy()
    cq = lay["cu_q"]
    words = [otree.ancestor_words(pp[cq[b]:cq[b + 1]]) for b in range(w.B)]
    expect = oattn.tree_attention(q.float().cpu(), k.float().cpu(), v.float().cpu(), lay["cu_q"], lay["cu_kv"],
                                  lay["prefix_len"], lay["pack_len"], words)
    e_ours = (ours.float().cpu() - expect).abs().max().item()
    e_ref = (theirs.float().cpu() - expect).abs().max().item()
    assert e_ours < (1e-4 if dtype == torch.float32 else 2e-2), e_ours
    assert e_ref < 5e-2, e_ref
    if dtype != torch.float32:
        assert (ours.float() - theirs.float()).abs().max().item() < 2e-2
