"""Run one kernel of the path on a benchmark configuration, for profilers.

    python -m cast_b200.bench_case --what attn --config 3 --batch 32 --iters 3
    python -m cast_b200.bench_case --what attn_store --config 3 --batch 32 --iters 3
    python -m cast_b200.bench_case --what topk --config 3 --batch 32 --iters 3
    python -m cast_b200.bench_case --what tree --config 3 --batch 32 --iters 3

Builds the first `batch` sequences of the configuration (trees from the GPU
tree builder), launches the chosen kernel `iters` times on one GPU and prints
the mean CUDA-event time per launch. `attn_store` runs the same attention with
the prefixes read in place from per-request stores [B, H_kv, S_max, D] and the
pack K/V as strided [T, H_kv, D] views of [H_kv, T, D] tensors. Meant to be wrapped by ncu with a kernel
filter (`-k regex:attn_tc|block_topk|build_tree`).
"""
import argparse
import json

import torch

import cast_b200
from cast_b200 import _lib, workloads


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--what", choices=["attn", "attn_store", "topk", "tree"], default="attn")
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
    if args.what == "attn_store":
        s_max = (max(w.S) + 255) // 256 * 256
        k_store = torch.zeros((w.B, w.H_kv, s_max, w.D), dtype=k.dtype, device=dev)
        v_store = torch.zeros_like(k_store)
        k_pack = torch.empty((w.H_kv, lay["total_q"], w.D), dtype=k.dtype, device=dev)
        v_pack = torch.empty_like(k_pack)
        for b in range(w.B):
            a, s_b, p_b, q0 = int(lay["cu_kv"][b]), w.S[b], int(lay["pack_len"][b]), int(lay["cu_q"][b])
            k_store[b, :, :s_b] = k[a:a + s_b].transpose(0, 1)
            v_store[b, :, :s_b] = v[a:a + s_b].transpose(0, 1)
            k_pack[:, q0:q0 + p_b] = k[a + s_b:a + s_b + p_b].transpose(0, 1)
            v_pack[:, q0:q0 + p_b] = v[a + s_b:a + s_b + p_b].transpose(0, 1)
        del k, v
        args_store = (q, k_store, v_store, k_pack.transpose(0, 1), v_pack.transpose(0, 1), t(lay["cu_q"]),
                      t(lay["prefix_len"]), t(lay["pack_len"]), None)

    def once():
        if args.what == "attn":
            cast_b200.varlen_tree_attention(*args_attn, parent=trees.pack_parent, max_pack=lay["max_pack"],
                                            max_kv=lay["max_kv"], out=out)
        elif args.what == "attn_store":
            cast_b200.varlen_tree_attention_store(*args_store, parent=trees.pack_parent, max_pack=lay["max_pack"],
                                                  max_prefix=max(w.S), out=out)
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
