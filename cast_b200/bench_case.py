"""Run one kernel of the path on a benchmark configuration, for profilers.

    python -m cast_b200.bench_case --what attn --config 3 --batch 32 --iters 3
    python -m cast_b200.bench_case --what topk --config 3 --batch 32 --iters 3
    python -m cast_b200.bench_case --what tree --config 3 --batch 32 --iters 3

Builds the first `batch` sequences of the configuration (trees from the GPU
tree builder), launches the chosen kernel `iters` times on one GPU and prints
the mean CUDA-event time per launch. Meant to be wrapped by ncu with a kernel
filter (`-k regex:attn_tc|block_topk|build_tree`).
"""
import argparse
import json

import torch

import cast_b200
from cast_b200 import _lib, workloads


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--what", choices=["attn", "topk", "tree"], default="attn")
    ap.add_argument("--config", type=int, default=3)
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--dtype", choices=["bf16", "fp16", "fp32"], default="bf16")
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    dtype = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[args.dtype]
    w = workloads.config(args.config, dtype)
    w = w.shard(list(range(min(args.batch, w.B))))
    lay = w.layout()
    logits = torch.from_numpy(w.logits_batch()).to(dev)
    idx, lp = cast_b200.block_topk_device(logits, 8)
    t = lambda a: torch.from_numpy(a).to(dev)
    budget = torch.tensor(w.N, dtype=torch.int32, device=dev)
    cu_q = t(lay["cu_q"])
    trees = cast_b200.build_trees(idx, lp, budget, 8, max_budget=max(w.N), cu_q=cu_q, total_q=lay["total_q"])
    q, k, v = w.make_qkv(dev)
    out = torch.empty_like(q)
    args_attn = (q, k, v, t(lay["cu_q"]), t(lay["cu_kv"]), t(lay["prefix_len"]), t(lay["pack_len"]), None)

    def once():
        if args.what == "attn":
            cast_b200.varlen_tree_attention(*args_attn, parent=trees.pack_parent, max_pack=lay["max_pack"],
                                            max_kv=lay["max_kv"], out=out)
        elif args.what == "topk":
            cast_b200.block_topk_device(logits, 8, idx, lp)
        else:
            cast_b200.build_trees(idx, lp, budget, 8, max_budget=max(w.N), cu_q=cu_q, total_q=lay["total_q"])

    once()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ev[0].record()
    for _ in range(args.iters):
        once()
    ev[1].record()
    torch.cuda.synchronize()
    if _lib.device_error() != 0:
        raise RuntimeError("device error")
    print(json.dumps({"what": args.what, "config": args.config, "batch": w.B,
                      "us_per_launch": round(ev[0].elapsed_time(ev[1]) * 1e3 / args.iters, 1)}))


if __name__ == "__main__":
    main()
