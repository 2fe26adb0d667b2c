"""CPU oracle for ragged ancestor-masked tree attention (test infrastructure only).

Restates the per-sequence fp32 dense reference of tests/test_tree_attn.py:40-59
for general pack sizes: sequence b owns keys concat(prefix_b, pack_b) at
cu_kv[b] (the pack starts at cu_kv[b] + prefix_len[b], tree_attn.py:71); a
query row sees every prefix key and the pack keys whose bit is set in its
ancestor bitset. Rows that see nothing return 0 (tree_attn.py:89). GQA maps
query head h to key/value head h // (H_q // H_kv) (tree_attn.py:30).
"""
import math

import numpy as np
import torch


def _visible_pack(words, P):
    """bool [P, P] from uint64/int64 ancestor words [P, W]."""
    w = np.asarray(words).view(np.uint64).reshape(P, -1)
    cols = np.arange(P)
    return ((w[:, cols // 64] >> (cols % 64).astype(np.uint64)) & np.uint64(1)).astype(bool)


def tree_attention(q, k, v, cu_q, cu_kv, prefix_len, pack_len, anc_words, sm_scale=None):
    """fp32 reference output [total_q, H_q, D] (torch, CPU).

    q: [total_q, H_q, D]; k, v: [total_kv, H_kv, D] (any float dtype, upcast
    to fp32). anc_words: per sequence, uint64 [P_b, W_b] ancestor words (a
    list), or one int64 array [total_q] / [total_q, W] as the reference API
    takes it.
    """
    q = torch.as_tensor(q).float().cpu()
    k = torch.as_tensor(k).float().cpu()
    v = torch.as_tensor(v).float().cpu()
    total_q, H_q, D = q.shape
    H_kv = k.shape[1]
    G = H_q // H_kv
    scale = 1.0 / math.sqrt(D) if sm_scale is None else float(sm_scale)
    cu_q = [int(x) for x in np.asarray(cu_q)]
    cu_kv = [int(x) for x in np.asarray(cu_kv)]
    prefix_len = [int(x) for x in np.asarray(prefix_len)]
    pack_len = [int(x) for x in np.asarray(pack_len)]
    out = torch.zeros(total_q, H_q, D, dtype=torch.float32)
    for b in range(len(pack_len)):
        S, P = prefix_len[b], pack_len[b]
        if P == 0:
            continue
        if isinstance(anc_words, (list, tuple)):
            words = np.asarray(anc_words[b])
        else:
            words = np.asarray(anc_words)[cu_q[b]:cu_q[b] + P]
        vis = np.ones((P, S + P), dtype=bool)
        vis[:, S:] = _visible_pack(words.reshape(P, -1), P)
        mask = torch.from_numpy(vis)
        qb = q[cu_q[b]:cu_q[b] + P].permute(1, 0, 2).reshape(H_kv, G * P, D)
        kb = k[cu_kv[b]:cu_kv[b] + S + P].permute(1, 0, 2)
        vb = v[cu_kv[b]:cu_kv[b] + S + P].permute(1, 0, 2)
        att = torch.matmul(qb, kb.transpose(1, 2)) * scale          # [H_kv, G*P, S+P]
        att = att.view(H_kv, G, P, S + P).masked_fill(~mask, float("-inf"))
        prob = torch.softmax(att, dim=-1).nan_to_num(0.0)            # empty rows -> 0
        ob = torch.matmul(prob.view(H_kv, G * P, S + P), vb)        # [H_kv, G*P, D]
        out[cu_q[b]:cu_q[b] + P] = ob.view(H_q, P, D).permute(1, 0, 2)
    return out
