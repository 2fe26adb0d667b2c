"""Greedy tree walk on the GPU (drop-in for cast_trees/decode.py:85-103 at T=0).

``walk_trees_greedy`` walks every sequence of a packed verify pass in one
launch (the per-request loop of cast_trees/serving.py:326-336): from each
pack's root it takes the argmax of the current row's target logits, moves to
the child carrying that token (lowest node index first) and stops at the first
miss, whose token is the bonus. Only the rows on the accepted paths are read.

``walk_tree`` keeps the reference's per-tree signature for temperature 0.
"""
import ctypes
from typing import NamedTuple, Optional

import torch

from . import _lib

_DTYPES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


class Walk(NamedTuple):
    """Device result of walk_trees_greedy (row b = sequence b)."""
    path: torch.Tensor       # int32 [B, path_cap]: accepted node indices, -1 padded
    accepted: torch.Tensor   # int32 [B]: len(path) + 1
    bonus: torch.Tensor      # int64 [B]: token picked after the path
    keep: torch.Tensor       # int32 [B, path_cap + 1]: [0] + [i + 1 for i in path], -1 padded
    tokens: torch.Tensor     # int64 [B, path_cap + 1]: committed tokens (path tokens, bonus), -1 padded


def walk_trees_greedy(logits, cu_q, pack_parent, pack_token, path_cap, *, out: Optional[Walk] = None):
    """Greedy walk of every packed tree.

    logits: CUDA [total_q, V] (float32 / bfloat16 / float16, unit stride over
    V) in pack order; cu_q int32 [B+1]; pack_parent / pack_token int32
    [total_q] (pack-local parents with -1 at each root, and the token of every
    packed row, as build_trees writes them). path_cap bounds the accepted path
    length (max pack length - 1 always suffices). No device-to-host read.
    """
    if not logits.is_cuda:
        raise RuntimeError("cast_b200.walk_trees_greedy needs CUDA tensors (no CPU path)")
    if logits.dtype not in _DTYPES:
        logits = logits.float()
    if logits.dim() != 2 or logits.stride(-1) != 1:
        logits = logits.reshape(-1, logits.shape[-1]).contiguous()
    dev = logits.device
    as_i32 = lambda t: torch.as_tensor(t, device=dev).to(torch.int32).contiguous()
    cu_q, pack_parent, pack_token = as_i32(cu_q), as_i32(pack_parent), as_i32(pack_token)
    B = cu_q.numel() - 1
    path_cap = max(1, int(path_cap))
    if out is None:
        out = Walk(torch.empty((B, path_cap), dtype=torch.int32, device=dev),
                   torch.empty((B,), dtype=torch.int32, device=dev),
                   torch.empty((B,), dtype=torch.int64, device=dev),
                   torch.empty((B, path_cap + 1), dtype=torch.int32, device=dev),
                   torch.empty((B, path_cap + 1), dtype=torch.int64, device=dev))
    code = _lib.lib().cast_tree_walk_greedy(
        logits.data_ptr(), _DTYPES[logits.dtype], logits.stride(0), logits.shape[1], cu_q.data_ptr(),
        pack_parent.data_ptr(), pack_token.data_ptr(), B, logits.shape[0], path_cap, out.path.data_ptr(),
        out.accepted.data_ptr(), out.bonus.data_ptr(), out.keep.data_ptr(), out.tokens.data_ptr(),
        torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(code, "cast_tree_walk_greedy")
    return out


def walk_tree(nodes, logits, temperature=0.0, d_logits=None, draft_temp=1.0, generator=None):
    """(accepted path, next root token) of one verified tree, as cast_trees/decode.py:85-103.

    nodes: TreeNode list (token, depth, parent, score); logits: [1+N, V]
    target logits of the packed rows (root first). Temperature 0 only: the
    speculative-sampling branch (T > 0) is not part of this library.
    """
    if temperature >= 1e-5:
        raise NotImplementedError("cast_b200.walk_tree implements the greedy walk (temperature 0) only")
    if not isinstance(logits, torch.Tensor) or not logits.is_cuda:
        if not torch.cuda.is_available():
            raise RuntimeError("cast_b200.walk_tree needs a CUDA device (no CPU path)")
        logits = torch.as_tensor(logits).to(torch.device("cuda", torch.cuda.current_device()))
    dev = logits.device
    n = len(nodes)
    pack_parent = torch.tensor([-1] + [nd.parent + 1 for nd in nodes], dtype=torch.int32, device=dev)
    pack_token = torch.tensor([-1] + [nd.token for nd in nodes], dtype=torch.int32, device=dev)
    cu_q = torch.tensor([0, n + 1], dtype=torch.int32, device=dev)
    w = walk_trees_greedy(logits[: n + 1], cu_q, pack_parent, pack_token, max(1, n))
    _lib.raise_device_error("cast_tree_walk_greedy")
    acc = int(w.accepted[0].item())
    path = w.path[0, : acc - 1].cpu().tolist()
    return path, int(w.bonus[0].item())


def committed(walk: Walk):
    """Host lists (keep, accepted, bonus, new tokens) per sequence, as serving.py:326-336 builds them."""
    acc = walk.accepted.cpu().tolist()
    keep = walk.keep.cpu().tolist()
    toks = walk.tokens.cpu().tolist()
    bonus = walk.bonus.cpu().tolist()
    return ([k[:a] for k, a in zip(keep, acc)], acc, bonus, [t[:a] for t, a in zip(toks, acc)])
