"""This library's attention beside the reference's own Triton kernel, both against the CPU oracle (GPU).

The reference kernel (cast_trees/tree_attn.py:17-92) is imported unmodified from the reference package
installed beside the repo (baseline/_ref); without it the test is skipped. The reference autotunes it over
BLOCK_N in {64, 128}, num_stages in {1, 2} and num_warps in {2, 4, 8} (tree_attn.py:95-101) and keeps the
fastest; here the undecorated kernel runs under every one of those configurations on the same inputs
(configuration 1 in fp32 and bf16, the configuration-2 sequences with N <= 63 in bf16: it takes packs of
at most 64 tokens). Only this library's output is held to the path's bound (1e-4 fp32, 2e-2 bf16); the
reference's error per configuration is printed as one JSON line per case (run with -s to see them),
since on this GPU some of its configurations are far outside its own test's 5e-2.
"""
import json
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
def test_against_oracle_beside_reference_kernel(cuda, cfg, dtype):
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
    pp = trees.pack_parent.cpu().numpy()
    cq = lay["cu_q"]
    words = [otree.ancestor_words(pp[cq[b]:cq[b + 1]]) for b in range(w.B)]
    expect = oattn.tree_attention(q.float().cpu(), k.float().cpu(), v.float().cpu(), lay["cu_q"], lay["cu_kv"],
                                  lay["prefix_len"], lay["pack_len"], words)
    ours = cast_b200.varlen_tree_attention(q, k, v, cu_q, cu_kv, prefix, pack, None, parent=trees.pack_parent)
    ours_bits = cast_b200.varlen_tree_attention(q, k, v, cu_q, cu_kv, prefix, pack, bits)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    e_ours = (ours.float().cpu() - expect).abs().max().item()
    rows = [{"impl": "cast_b200", "max_abs_err": e_ours,
             "bits_and_parent_identical": bool(torch.equal(ours, ours_bits))}]
    req, row0, nrows = ref_ta._tile_schedule(cu_q.cpu(), cuda)
    for bn in (64, 128):
        for stages in (1, 2):
            for warps in (2, 4, 8):
                out = torch.zeros_like(q)
                ref_ta._tree_attn_fwd[(req.numel(), w.H_q)](
                    q, k, v, out, bits, req, row0, nrows, cu_kv, prefix, pack, 1.0 / (w.D ** 0.5),
                    q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2),
                    v.stride(0), v.stride(1), v.stride(2), out.stride(0), out.stride(1), out.stride(2),
                    H_q=w.H_q, GROUP=w.H_q // w.H_kv, D=w.D, BLOCK_M=ref_ta.BLOCK_M, BLOCK_N=bn,
                    num_stages=stages, num_warps=warps)
                torch.cuda.synchronize()
                err = (out.float().cpu() - expect).abs()
                rows.append({"impl": "reference triton", "BLOCK_N": bn, "num_stages": stages, "num_warps": warps,
                             "max_abs_err": err.max().item(), "rows_over_5e-2": int((err.amax(dim=2) > 5e-2).sum())})
    print(json.dumps({"what": "vs_triton_configs", "config": cfg, "dtype": str(dtype).replace("torch.", ""),
                      "batch": w.B, "rows": rows}))
    assert e_ours < (1e-4 if dtype == torch.float32 else 2e-2), e_ours
    assert rows[0]["bits_and_parent_identical"]
