"""Attention latency by tree width: the l(N) probe that feeds CAST's width rule.

    python -m cast_b200.width_probe --config 5 --batch 512 --iters 5

For each tree width N (default 16, 24, 32, 48, 64, 96, 128, 256) the probe
builds the N-node best-first tree of every sequence of the configuration on
the GPU (block_topk + build_tree over seeded normal(scale=5) block scores of
15 x V, drawn on the device), then times one ragged tree-attention call over
the whole batch (CUDA events, mean of `iters` after warm-up). It prints one
JSON object: the packed widths n = N + 1, the attention time per call (ms),
and the least-squares intercept and slope over 16 <= n <= 128 - the same fit
cast_trees/width.py:22-27 (fit_cost) makes - so the curve can be handed to
cast_trees.width.predict_width(n, ms). The slope c1 is the attention cost per
packed token for this batch, per layer.
"""
import argparse
import json

import numpy as np
import torch

import cast_b200
from cast_b200 import _lib, workloads

WIDTHS = (16, 24, 32, 48, 64, 96, 128, 256)


def probe(config=5, batch=512, widths=WIDTHS, iters=5, warmup=2, seed_offset=0, device=None):
    dev = device or torch.device("cuda", torch.cuda.current_device())
    base = workloads.config(config)
    base = base.shard(list(range(min(batch, base.B))))
    B, V = base.B, base.V
    g = torch.Generator(device=dev).manual_seed(base.seed * 7919 + seed_offset)
    logits = torch.empty((B, 15, V), dtype=torch.float64, device=dev)
    logits.normal_(generator=g).mul_(5.0)
    idx, lp = cast_b200.block_topk_device(logits, 8)
    del logits
    rows = []
    for N in widths:
        w = workloads.with_width(base, N)
        lay = w.layout()
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        cu_q = t(lay["cu_q"])
        trees = cast_b200.build_trees(idx, lp, N, 8, max_budget=N, cu_q=cu_q, total_q=lay["total_q"])
        q, k, v = w.make_qkv(dev)
        out = torch.empty_like(q)
        args = (q, k, v, cu_q, t(lay["cu_kv"]), t(lay["prefix_len"]), t(lay["pack_len"]), None)
        kw = dict(parent=trees.pack_parent, max_pack=lay["max_pack"], max_kv=lay["max_kv"], out=out)
        for _ in range(warmup):
            cast_b200.varlen_tree_attention(*args, **kw)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            cast_b200.varlen_tree_attention(*args, **kw)
        e1.record()
        torch.cuda.synchronize()
        if _lib.device_error() != 0:
            raise RuntimeError("device error during the width probe")
        ms = e0.elapsed_time(e1) / iters
        depth_sums = trees.depth.sum(dim=1, dtype=torch.int64).cpu().tolist()
        rows.append(dict(N=N, n=N + 1, ms=ms, tflops=w.attn_flops(depth_sums) / (ms * 1e-3) / 1e12))
        del q, k, v, out, trees
        torch.cuda.empty_cache()
    n = np.array([r["n"] for r in rows], dtype=float)
    ms = np.array([r["ms"] for r in rows], dtype=float)
    sel = (n >= 16) & (n <= 128)
    c1, c0 = np.polyfit(n[sel], ms[sel], 1)
    return dict(config=config, batch=B, widths=[r["N"] for r in rows], n=n.tolist(), ms=ms.tolist(),
                tflops=[round(r["tflops"], 1) for r in rows], c0_ms=float(c0), c1_ms_per_packed_token=float(c1))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", type=int, default=5)
    ap.add_argument("--batch", type=int, default=512)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--widths", default=",".join(str(x) for x in WIDTHS))
    args = ap.parse_args()
    widths = tuple(int(x) for x in args.widths.split(","))
    print(json.dumps(probe(args.config, args.batch, widths, args.iters)))


if __name__ == "__main__":
    main()
