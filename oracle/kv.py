"""CPU oracle for the KV-store steps of a verify round (test infrastructure only).

* ``append_store`` restates cast_trees/serving.py:264-289
  (BatchedServer._append_store) on numpy arrays.
* ``gather_cache`` restates cast_trees/verify.py:48-60 on numpy arrays.

Pinned by tests/golden/append.npz and gather.npz, which the reference itself
produced (tests/golden/make_golden.py).
"""
import numpy as np


def append_store(buf_k, buf_v, store_len, cu_q, keep, accepted, rows, pack_k, pack_v):
    """buf_*: per-layer [B, H, cap, D]; pack_*: per-layer [H, total_q, D]. Returns (k, v, new_len).

    Order of the reference: gather the surviving rows (serving.py:275-278),
    grow the capacity with zeros to max(max(new_len), 2 * cap) when needed
    (:279-282), then write pack row cu_q[b] + keep[b][j] at row
    store_len[b] + j of destination row nb (:283-288).
    """
    new_len = [store_len[b] + accepted[b] for b in rows]
    ks, vs = [np.array(x) for x in buf_k], [np.array(x) for x in buf_v]
    if len(rows) != len(store_len):
        ks = [x[list(rows)] for x in ks]
        vs = [x[list(rows)] for x in vs]
    cap = ks[0].shape[2]
    if max(new_len) > cap:
        new_cap = max(max(new_len), 2 * cap)
        grow = lambda x: np.concatenate([x, np.zeros(x.shape[:2] + (new_cap - cap,) + x.shape[3:], x.dtype)], 2)
        ks, vs = [grow(x) for x in ks], [grow(x) for x in vs]
    for li in range(len(ks)):
        for nb, b in enumerate(rows):
            for j, pk in enumerate(keep[b]):
                ks[li][nb, :, store_len[b] + j] = pack_k[li][:, cu_q[b] + pk]
                vs[li][nb, :, store_len[b] + j] = pack_v[li][:, cu_q[b] + pk]
    return ks, vs, new_len


def gather_cache(ks, vs, n_prefix, keep):
    """Per-layer [B, H, S, D] -> [B, H, n_prefix + len(keep), D]: the prefix, then rows n_prefix + keep[j]."""
    sel = list(range(n_prefix)) + [n_prefix + i for i in (keep or [])]
    return [np.array(k)[:, :, sel] for k in ks], [np.array(v)[:, :, sel] for v in vs]
