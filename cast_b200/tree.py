"""Best-first candidate trees on the GPU (drop-in for cast_trees/tree.py).

``block_topk`` and ``build_tree`` keep the reference's signatures, tie rules
and node order (cast_trees/tree.py:20-49) and run on the device through the C
ABI. ``build_trees`` is the batched device form used on the verify path: one
launch builds every sequence's tree and, optionally, the packed layout the
attention call consumes (pack-local parents, tokens, positions;
cast_trees/serving.py:213-222).
"""
import ctypes
from dataclasses import dataclass
from typing import NamedTuple, Optional

import numpy as np
import torch

from . import _lib


@dataclass
class TreeNode:
    """Field-for-field the reference's node (cast_trees/tree.py:12-17)."""
    token: int
    depth: int      # offset from the pending root, 1..L
    parent: int     # index into the node list, -1 = root
    score: float    # path log-probability under the drafter marginals


class Trees(NamedTuple):
    """Device result of build_trees: row b holds count[b] nodes in pop order."""
    token: torch.Tensor    # int32 [B, max_budget]
    depth: torch.Tensor    # int32 [B, max_budget]
    parent: torch.Tensor   # int32 [B, max_budget] (tree-local, -1 = root)
    score: torch.Tensor    # float64 [B, max_budget]
    count: torch.Tensor    # int32 [B]
    pack_parent: Optional[torch.Tensor] = None   # int32 [total_q], pack-local
    pack_token: Optional[torch.Tensor] = None    # int32 [total_q]
    pack_pos: Optional[torch.Tensor] = None      # int32 [total_q]
    cu_q: Optional[torch.Tensor] = None          # int32 [B+1] (select_global_topk_device output)


def _stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


def _cuda_device():
    if not torch.cuda.is_available():
        raise RuntimeError("cast_b200 tree construction needs a CUDA device (no CPU path)")
    return torch.device("cuda", torch.cuda.current_device())


def block_topk_device(logits, k=8, out_idx=None, out_lp=None):
    """Top-k of the fp64 log-softmax of every row of a CUDA tensor [..., V].

    Returns (idx int64 [..., k], lp float64 [..., k]) on the same device.
    """
    if logits.dtype != torch.float64:
        logits = logits.to(torch.float64)
    V = logits.shape[-1]
    lead = logits.shape[:-1]
    x = logits.reshape(-1, V)
    if x.stride(-1) != 1:
        x = x.contiguous()
    rows = x.shape[0]
    idx = out_idx if out_idx is not None else torch.empty((*lead, k), dtype=torch.int64, device=x.device)
    lp = out_lp if out_lp is not None else torch.empty((*lead, k), dtype=torch.float64, device=x.device)
    code = _lib.lib().cast_block_topk(x.data_ptr(), rows, V, x.stride(0), k, idx.data_ptr(), lp.data_ptr(),
                                      _stream(x.device))
    _lib.check(code, "cast_block_topk")
    return idx, lp


def block_topk(logits, k=8):
    """Top-k token ids and log-probs at each of the L future positions.

    Same contract as cast_trees/tree.py:20-26: numpy in, numpy out (computed
    on the GPU); a CUDA tensor in gives CUDA tensors out.
    """
    if isinstance(logits, torch.Tensor) and logits.is_cuda:
        return block_topk_device(logits, k)
    dev = _cuda_device()
    x = torch.as_tensor(np.asarray(logits, dtype=np.float64)).to(dev)
    idx, lp = block_topk_device(x, k)
    _lib.raise_device_error("cast_block_topk")
    return idx.cpu().numpy(), lp.cpu().numpy()


def build_trees(top_idx, top_lp, budget, k=8, *, max_budget=None, cu_q=None, root_token=None,
                seq_len=None, total_q=None):
    """Batched best-first trees on the device.

    top_idx int64 [B, L, kc], top_lp float64 [B, L, kc] (CUDA); budget: int or
    int32 [B]. With cu_q (int32 [B+1]) the pack-local parent array of each
    pack is written at its rows; root_token / seq_len add the packed tokens
    and positions. Pass total_q (= cu_q[-1]) and, for a tensor budget,
    max_budget to keep the call free of device-to-host reads.
    """
    dev = top_idx.device
    B, L, kc = top_idx.shape
    if isinstance(budget, int):
        mb = budget if max_budget is None else max_budget
        budget_t = torch.full((B,), budget, dtype=torch.int32, device=dev)
    else:
        budget_t = torch.as_tensor(budget, device=dev).to(torch.int32).contiguous()
        mb = int(budget_t.max().item()) if max_budget is None else max_budget
    top_idx = top_idx.contiguous()
    top_lp = top_lp.to(torch.float64).contiguous()
    token = torch.empty((B, max(mb, 1)), dtype=torch.int32, device=dev)
    depth = torch.empty_like(token)
    parent = torch.empty_like(token)
    score = torch.empty((B, max(mb, 1)), dtype=torch.float64, device=dev)
    count = torch.empty((B,), dtype=torch.int32, device=dev)
    pack_parent = pack_token = pack_pos = None
    cu_ptr = rt_ptr = sl_ptr = None
    if cu_q is not None:
        cu_q = torch.as_tensor(cu_q, device=dev).to(torch.int32).contiguous()
        if total_q is None:
            total_q = int(cu_q[-1].item())
        cu_ptr = cu_q.data_ptr()
        pack_parent = torch.empty(total_q, dtype=torch.int32, device=dev)
        if root_token is not None:
            root_token = torch.as_tensor(root_token, device=dev).to(torch.int32).contiguous()
            rt_ptr = root_token.data_ptr()
            pack_token = torch.empty(total_q, dtype=torch.int32, device=dev)
        if seq_len is not None:
            seq_len = torch.as_tensor(seq_len, device=dev).to(torch.int32).contiguous()
            sl_ptr = seq_len.data_ptr()
            pack_pos = torch.empty(total_q, dtype=torch.int32, device=dev)
    ptr = lambda t: None if t is None else t.data_ptr()
    code = _lib.lib().cast_build_tree(
        top_idx.data_ptr(), top_lp.data_ptr(), B, L, kc, k, budget_t.data_ptr(), mb,
        token.data_ptr(), depth.data_ptr(), parent.data_ptr(), score.data_ptr(), count.data_ptr(),
        cu_ptr, ptr(pack_parent), rt_ptr, ptr(pack_token), sl_ptr, ptr(pack_pos), _stream(dev))
    _lib.check(code, "cast_build_tree")
    return Trees(token, depth, parent, score, count, pack_parent, pack_token, pack_pos)


def build_tree(top_idx, top_lp, budget, k=8):
    """Best-first prefix-closed tree with `budget` nonroot nodes (list of TreeNode).

    Same contract and node order as cast_trees/tree.py:29-49; computed on the
    GPU. top_idx / top_lp: (L, >=k) arrays or tensors.
    """
    dev = _cuda_device()
    idx = torch.as_tensor(np.asarray(top_idx) if not isinstance(top_idx, torch.Tensor) else top_idx)
    lp = torch.as_tensor(np.asarray(top_lp, dtype=np.float64) if not isinstance(top_lp, torch.Tensor)
                         else top_lp)
    idx = idx.to(dev, torch.int64)[None]
    lp = lp.to(dev, torch.float64)[None]
    t = build_trees(idx, lp, int(budget), k)
    _lib.raise_device_error("cast_build_tree")
    n = int(t.count[0].item())
    tok, dep, par = (x[0, :n].cpu().tolist() for x in (t.token, t.depth, t.parent))
    sc = t.score[0, :n].cpu().tolist()
    return [TreeNode(int(a), int(b), int(c), float(d)) for a, b, c, d in zip(tok, dep, par, sc)]


def select_global_topk_device(trees: Trees, total, *, root_token=None, seq_len=None, pack_capacity=None):
    """Shared-budget split of a device forest (cast_trees/tree.py:63-82), in one launch.

    trees: a Trees from build_trees. The `total` best nodes of the pooled
    forest by (-score, tree, node) are kept; each tree keeps its nodes in
    order with renumbered parents. The result is a Trees of the same width
    with the new counts and, always, the packed layout of the selected trees
    (cu_q [B+1], pack_parent, and pack_token / pack_pos when root_token /
    seq_len are given). pack_capacity (default B + min(total, B * width))
    sizes the pack arrays without a device-to-host read.
    """
    token, depth, parent, score, count = trees.token, trees.depth, trees.parent, trees.score, trees.count
    dev = token.device
    B, mb = token.shape
    total = int(total)
    if pack_capacity is None:
        tot = total if total >= 0 else B * mb
        pack_capacity = B + max(0, min(tot, B * mb))
    o = [torch.empty_like(token), torch.empty_like(depth), torch.empty_like(parent), torch.empty_like(score),
         torch.empty_like(count)]
    cu_q = torch.empty((B + 1,), dtype=torch.int32, device=dev)
    pack_parent = torch.empty((max(1, pack_capacity),), dtype=torch.int32, device=dev)
    pack_token = pack_pos = None
    rt_ptr = sl_ptr = None
    if root_token is not None:
        root_token = torch.as_tensor(root_token, device=dev).to(torch.int32).contiguous()
        rt_ptr = root_token.data_ptr()
        pack_token = torch.empty_like(pack_parent)
    if seq_len is not None:
        seq_len = torch.as_tensor(seq_len, device=dev).to(torch.int32).contiguous()
        sl_ptr = seq_len.data_ptr()
        pack_pos = torch.empty_like(pack_parent)
    ptr = lambda t: None if t is None else t.data_ptr()
    code = _lib.lib().cast_select_global_topk(
        token.data_ptr(), depth.data_ptr(), parent.data_ptr(), score.data_ptr(), count.data_ptr(), B, mb, total,
        o[0].data_ptr(), o[1].data_ptr(), o[2].data_ptr(), o[3].data_ptr(), o[4].data_ptr(), cu_q.data_ptr(),
        rt_ptr, sl_ptr, pack_parent.data_ptr(), ptr(pack_token), ptr(pack_pos), int(pack_capacity),
        _stream(dev))
    _lib.check(code, "cast_select_global_topk")
    return Trees(o[0], o[1], o[2], o[3], o[4], pack_parent, pack_token, pack_pos, cu_q)


def select_global_topk(trees, total):
    """Split a shared budget across requests by global best-first score.

    Same contract as cast_trees/tree.py:63-82: a list of TreeNode lists in,
    a list of TreeNode lists out (the first `total` nodes of the pool sorted
    by (-score, request, node) are kept, in node order, parents renumbered);
    computed on the GPU.
    """
    B = len(trees)
    if B == 0:
        return []
    dev = _cuda_device()
    mb = max(1, max(len(t) for t in trees))
    tok = np.zeros((B, mb), dtype=np.int32)
    dep = np.zeros((B, mb), dtype=np.int32)
    par = np.full((B, mb), -1, dtype=np.int32)
    sc = np.zeros((B, mb), dtype=np.float64)
    cnt = np.array([len(t) for t in trees], dtype=np.int32)
    for b, nodes in enumerate(trees):
        for j, nd in enumerate(nodes):
            tok[b, j], dep[b, j], par[b, j], sc[b, j] = nd.token, nd.depth, nd.parent, nd.score
    t = lambda a: torch.from_numpy(a).to(dev)
    src = Trees(t(tok), t(dep), t(par), t(sc), t(cnt))
    out = select_global_topk_device(src, total)
    _lib.raise_device_error("cast_select_global_topk")
    n = out.count.cpu().tolist()
    tok, dep, par, sc = (x.cpu().tolist() for x in (out.token, out.depth, out.parent, out.score))
    return [[TreeNode(int(tok[b][i]), int(dep[b][i]), int(par[b][i]), float(sc[b][i])) for i in range(n[b])]
            for b in range(B)]
