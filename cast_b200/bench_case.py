"""Run one kernel of the path on a benchmark configuration, for profilers.

    python -m cast_b200.bench_case --what attn --config 3 --batch 32 --iters 3
    python -m cast_b200.bench_case --what attn_store --config 3 --batch 32 --iters 3
    python -m cast_b200.bench_case --what topk --config 3 --batch 32 --iters 3
    python -m cast_b200.bench_case --what tree --config 3 --batch 32 --iters 3
    python -m cast_b200.bench_case --what walk --config 3 --batch 64 --iters 20
    python -m cast_b200.bench_case --what select --config 5 --batch 512 --iters 20
    python -m cast_b200.bench_case --what append --config 3 --batch 64 --iters 20

    python -m cast_b200.bench_case --what vs_triton --config 1
    python -m cast_b200.bench_case --what vs_triton --config 2
    python -m cast_b200.bench_case --what vs_triton --config 0
    python -m cast_b200.bench_case --what vs_triton --config 5 --batch 64 --width 32

Builds the first `batch` sequences of the configuration (trees from the GPU
tree builder), launches the chosen kernel `iters` times on one GPU and prints
the mean CUDA-event time per launch. `attn_store` runs the same attention with
the prefixes read in place from per-request stores [B, H_kv, S_max, D] and the
pack K/V as strided [T, H_kv, D] views of [H_kv, T, D] tensors. `walk` runs
the greedy walk over synthetic bf16 target logits [total_q, V] that follow each
tree for a few levels; `select` splits a shared budget of 8 nodes per request
over trees built at width 48; `append` appends each walk's accepted rows to
32 layers of per-request stores in place. Meant to be wrapped by ncu with a kernel
filter (`-k regex:attn_tc|block_topk|build_tree`).

`vs_triton` times this library's attention against the reference's own GPU
kernel (cast_trees/tree_attn.py:116-139, the Triton `_tree_attn_fwd`, imported
unmodified from the reference package installed beside the repo in
baseline/_ref) on the same inputs. That kernel takes packs of at most 64
tokens (one int64 ancestor word per row), so it runs configuration 1 (fp32 and
bf16), the configuration-2 sequences with N <= 63, and configuration 5 at one
width N <= 63 (`--width`, on a batch small enough for the reference kernel's
32-bit element offsets: 64 sequences); `--config 0` runs the reference test's
own scenario. Both are timed through their public calls (the
reference's reads cu_q back to the host every call) and the reference's kernel
also alone, on a precomputed tile schedule.
"""
import argparse
import json

import numpy as np
import torch

import cast_b200
from cast_b200 import _lib, workloads


def _ancestor_bits(pack_parent, cu_q, pack_len, max_depth):
    """int64 [total_q] ancestor bitmask of every pack token (bit j = pack index j), pack index < 64.

    Equivalent of the reference's host loop (cast_trees/serving.py:213-222): a token's word is its
    own bit or'ed with its parent's word, built here by walking up at most `max_depth` levels.
    """
    dev = pack_parent.device
    total_q = pack_parent.shape[0]
    q0 = torch.repeat_interleave(cu_q[:-1].long(), pack_len.long(), output_size=total_q)
    local = torch.arange(total_q, device=dev) - q0
    bits = torch.bitwise_left_shift(torch.ones_like(local), local)
    cur = pack_parent.long()
    for _ in range(max_depth + 1):
        live = cur >= 0
        if not bool(live.any()):
            break
        bits = torch.where(live, bits | torch.bitwise_left_shift(torch.ones_like(cur), cur.clamp(min=0)), bits)
        cur = torch.where(live, pack_parent.long()[(q0 + cur.clamp(min=0))], cur)
    return bits


def _event_us(fn, iters):
    fn()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ev[0].record()
    for _ in range(iters):
        fn()
    ev[1].record()
    torch.cuda.synchronize()
    return ev[0].elapsed_time(ev[1]) * 1e3 / iters


def _ref_offsets_unsafe(total_q, total_kv, H_q, H_kv, D):
    """Why the reference kernel must not run on these sizes, or None.

    Its element offsets (row * stride, cast_trees/tree_attn.py:44-58) are 32-bit; a tensor of 2^31
    elements or more overflows them and the kernel reads out of bounds (on this pool it raised an
    illegal memory access on configuration 5's 4.8e9-element K/V).
    """
    if max(total_q * H_q * D, total_kv * H_kv * D) >= 2 ** 31:
        return ("q/k/v hold 2^31 elements or more: the reference kernel's 32-bit offsets overflow "
                "(illegal memory access on this pool); use a smaller --batch")
    return None


def vs_triton_scenario(args, dev, ref_ta):
    """The reference test's own scenario (cast_trees tests/test_tree_attn.py:11-37 shape: B=8, 32/8 heads,
    D=128, S in [200, 400), P in [2, 64), uniform random parents, N(0,1) inputs) through both kernels."""
    g = torch.Generator().manual_seed(0)
    qs, ks, vs, bits, S, P, cu_q, cu_kv = [], [], [], [], [], [], [0], [0]
    for _ in range(8):
        s_b = int(torch.randint(200, 400, (1,), generator=g))
        p_b = int(torch.randint(2, 64, (1,), generator=g))
        parent = [-1] + [int(torch.randint(0, i, (1,), generator=g)) for i in range(1, p_b)]
        qs.append(torch.randn(p_b, 32, 128, generator=g))
        ks.append(torch.randn(s_b + p_b, 8, 128, generator=g))
        vs.append(torch.randn(s_b + p_b, 8, 128, generator=g))
        for i in range(p_b):
            wd, j = 0, i
            while j != -1:
                wd |= 1 << j
                j = parent[j]
            bits.append(wd)
        S.append(s_b)
        P.append(p_b)
        cu_q.append(cu_q[-1] + p_b)
        cu_kv.append(cu_kv[-1] + s_b + p_b)
    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device=dev)
    cu_q_t, cu_kv_t, pre, pk = i32(cu_q), i32(cu_kv), i32(S), i32(P)
    bits_t = torch.tensor(np.array(bits, dtype=np.uint64).view(np.int64), device=dev)
    rows = []
    for dtype in (torch.float32, torch.bfloat16):
        q, k, v = (torch.cat(x).to(dev, dtype) for x in (qs, ks, vs))
        o_ref = ref_ta.varlen_tree_attention(q, k, v, cu_q_t, cu_kv_t, pre, pk, bits_t)
        o_ours = cast_b200.varlen_tree_attention(q, k, v, cu_q_t, cu_kv_t, pre, pk, bits_t)
        torch.cuda.synchronize()
        if _lib.device_error() != 0:
            raise RuntimeError("device error")
        rows.append({"dtype": str(dtype).replace("torch.", ""),
                     "max_abs_diff_ours_vs_ref": (o_ours.float() - o_ref.float()).abs().max().item(),
                     "mean_abs_diff_ours_vs_ref": (o_ours.float() - o_ref.float()).abs().mean().item()})
    print(json.dumps({"what": "vs_triton", "config": 0, "case": "reference test scenario (seed 0)", "rows": rows}))


def vs_triton(args, dev):
    """This library's tree attention against the reference's Triton kernel on the same inputs."""
    import sys
    from pathlib import Path
    ref_dir = Path(__file__).resolve().parent.parent / "baseline" / "_ref"
    if not (ref_dir / "cast_trees" / "tree_attn.py").exists():
        print(json.dumps({"what": "vs_triton", "unavailable": "reference package not installed in baseline/_ref"}))
        return
    sys.path.insert(0, str(ref_dir))
    from cast_trees import tree_attn as ref_ta
    dtypes = {"bf16": [torch.bfloat16], "fp16": [torch.float16], "fp32": [torch.float32]}[args.dtype]
    if args.config == 1:
        dtypes = [torch.float32, torch.bfloat16]
    if args.config == 0:
        return vs_triton_scenario(args, dev, ref_ta)
    base = workloads.config(args.config)
    if args.config == 5:
        base = workloads.with_width(base.shard(list(range(min(args.batch, base.B)))), args.width)
    elif args.config == 2:
        base = base.shard([b for b in range(base.B) if base.N[b] <= 63])
    w = base
    assert max(w.P) <= 64, "the reference kernel takes packs of at most 64 tokens"
    lay = w.layout()
    why = _ref_offsets_unsafe(lay["total_q"], lay["total_kv"], w.H_q, w.H_kv, w.D)
    if why:
        print(json.dumps({"what": "vs_triton", "config": args.config, "batch": w.B, "unavailable": why}))
        return
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    if args.config == 5:
        g = torch.Generator(device=dev).manual_seed(w.seed * 7919 + 17)
        logits = torch.empty((w.B, 15, w.V), dtype=torch.float64, device=dev).normal_(generator=g).mul_(5.0)
    else:
        logits = t(w.logits_batch())
    idx, lp = cast_b200.block_topk_device(logits, 8)
    del logits
    cu_q, cu_kv, prefix, pack = t(lay["cu_q"]), t(lay["cu_kv"]), t(lay["prefix_len"]), t(lay["pack_len"])
    budget = torch.tensor(w.N, dtype=torch.int32, device=dev)
    trees = cast_b200.build_trees(idx, lp, budget, 8, max_budget=max(w.N), cu_q=cu_q, total_q=lay["total_q"])
    bits = _ancestor_bits(trees.pack_parent, cu_q, pack, 15)
    rows = []
    for dtype in dtypes:
        q, k, v = w.make_qkv(dev, dtype)
        out = torch.empty_like(q)
        ours = lambda: cast_b200.varlen_tree_attention(q, k, v, cu_q, cu_kv, prefix, pack, None,
                                                       parent=trees.pack_parent, max_pack=lay["max_pack"],
                                                       max_kv=lay["max_kv"], out=out)
        theirs = lambda: ref_ta.varlen_tree_attention(q, k, v, cu_q, cu_kv, prefix, pack, bits)
        o_ref = theirs()                  # first call autotunes the Triton kernel
        torch.cuda.synchronize()
        o_ours = ours().clone()
        o_bits = cast_b200.varlen_tree_attention(q, k, v, cu_q, cu_kv, prefix, pack, bits,
                                                 max_pack=lay["max_pack"], max_kv=lay["max_kv"])
        if _lib.device_error() != 0:
            raise RuntimeError("device error")
        us_ours = _event_us(ours, args.iters)
        us_ref = _event_us(theirs, args.iters)
        req, row0, nrows = ref_ta._tile_schedule(cu_q.cpu(), dev)
        sm_scale = 1.0 / (w.D ** 0.5)
        out_k = torch.empty_like(q)

        def ref_kernel():
            ref_ta._tree_attn[(req.numel(), w.H_q)](
                q, k, v, out_k, bits, req, row0, nrows, cu_kv, prefix, pack, sm_scale,
                q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2),
                v.stride(0), v.stride(1), v.stride(2), out_k.stride(0), out_k.stride(1), out_k.stride(2),
                H_q=w.H_q, GROUP=w.H_q // w.H_kv, D=w.D, BLOCK_M=ref_ta.BLOCK_M)
        us_ref_k = _event_us(ref_kernel, args.iters)
        depth_sums = trees.depth.sum(dim=1, dtype=torch.int64).cpu().tolist()
        fl = w.attn_flops(depth_sums)
        kernel, n_split, _ = cast_b200.attention_plan(q, k, v, out, w.B, lay["max_pack"], lay["max_kv"])
        rows.append({"dtype": str(dtype).replace("torch.", ""), "kernel": kernel, "key_splits": n_split,
                     "us_ours": round(us_ours, 1), "us_ref_api": round(us_ref, 1), "us_ref_kernel": round(us_ref_k, 1),
                     "speedup_vs_ref_api": round(us_ref / us_ours, 2),
                     "speedup_vs_ref_kernel": round(us_ref_k / us_ours, 2),
                     "tflops_ours": round(fl / (us_ours * 1e-6) / 1e12, 2),
                     "tflops_ref_kernel": round(fl / (us_ref_k * 1e-6) / 1e12, 2),
                     "max_abs_diff_ours_vs_ref": (o_ours.float() - o_ref.float()).abs().max().item(),
                     "bits_and_parent_identical": bool(torch.equal(o_ours, o_bits))})
        del q, k, v, out, out_k
    print(json.dumps({"what": "vs_triton", "config": args.config, "batch": w.B,
                      "width": args.width if args.config == 5 else None,
                      "P": sorted(set(w.P)), "S_range": [min(w.S), max(w.S)], "rows": rows}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--what", choices=["attn", "attn_store", "topk", "tree", "walk", "select", "append", "vs_triton"],
                    default="attn")
    ap.add_argument("--width", type=int, default=32, help="vs_triton on configuration 5: tree width N (<= 63)")
    ap.add_argument("--config", type=int, default=3)
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--dtype", choices=["bf16", "fp16", "fp32"], default="bf16")
    ap.add_argument("--graph", action="store_true",
                    help="also time the calls replayed from a CUDA graph (device time without host overhead)")
    ap.add_argument("--kernel", choices=["auto", "single", "simt"], default="auto",
                    help="16-bit attention kernel: the library's choice (CTA pairs where they apply), "
                         "single-CTA tcgen05 always, or the CUDA-core kernel (to measure the dispatch)")
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    _lib.lib().cast_test_set_tc_kernel({"auto": 1, "single": 0, "simt": -1}[args.kernel])
    if args.what == "vs_triton":
        vs_triton(args, dev)
        return
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

    if args.what in ("walk", "append"):
        gen = torch.Generator(device=dev).manual_seed(7)
        tl = torch.empty((lay["total_q"], w.V), dtype=torch.bfloat16, device=dev)
        tl.normal_(generator=gen)
        pp, ptok = trees.pack_parent, torch.zeros_like(trees.pack_parent)
        # tokens: node tokens (root 0); plant the first child's token as each row's argmax
        ptok = torch.where(pp >= 0, torch.randint(0, w.V, ptok.shape, device=dev, dtype=torch.int32), ptok)
        rows = torch.arange(lay["total_q"], device=dev)
        big = torch.iinfo(torch.int64).max
        first_child = torch.full((lay["total_q"],), big, dtype=torch.int64, device=dev)
        q0 = torch.repeat_interleave(t(lay["cu_q"][:-1]).long(), t(lay["pack_len"]).long())
        par_abs = torch.where(pp >= 0, q0 + pp.long(), torch.full_like(q0, -1))
        child_rows = rows[par_abs >= 0]
        first_child.scatter_reduce_(0, par_abs[child_rows], child_rows, reduce="amin")
        # a row follows its first child with probability 3/4 (mean accepted length near 4)
        has = (first_child < big) & (torch.rand(first_child.shape, generator=gen, device=dev) < 0.75)
        tl[rows[has], ptok[first_child[has]].long()] = 50.0
        path_cap = lay["max_pack"] - 1
        walk_out = cast_b200.walk_trees_greedy(tl, cu_q, pp, ptok, path_cap)
    if args.what == "append":
        n_layers, s_cap = 32, (max(w.S) + 320 + 255) // 256 * 256
        sl_t = t(lay["prefix_len"])
        mk = lambda: torch.zeros((w.B, w.H_kv, s_cap, w.D), dtype=torch.bfloat16, device=dev)
        bk = [mk() for _ in range(n_layers)]
        bv = [mk() for _ in range(n_layers)]
        pk = [torch.randn((w.H_kv, lay["total_q"], w.D), device=dev).to(torch.bfloat16) for _ in range(n_layers)]
        pv = [torch.randn((w.H_kv, lay["total_q"], w.D), device=dev).to(torch.bfloat16) for _ in range(n_layers)]
    if args.what == "select":
        sel_src = cast_b200.build_trees(idx, lp, 48, 8, max_budget=48)

    def once():
        if args.what == "attn":
            cast_b200.varlen_tree_attention(*args_attn, parent=trees.pack_parent, max_pack=lay["max_pack"],
                                            max_kv=lay["max_kv"], out=out)
        elif args.what == "attn_store":
            cast_b200.varlen_tree_attention_store(*args_store, parent=trees.pack_parent, max_pack=lay["max_pack"],
                                                  max_prefix=max(w.S), out=out)
        elif args.what == "topk":
            cast_b200.block_topk_device(logits, 8, idx, lp)
        elif args.what == "walk":
            cast_b200.walk_trees_greedy(tl, cu_q, pp, ptok, path_cap, out=walk_out)
        elif args.what == "select":
            cast_b200.select_global_topk_device(sel_src, 8 * w.B, pack_capacity=w.B * 9)
        elif args.what == "append":
            cast_b200.append_store_inplace(bk, bv, sl_t, cu_q[:-1], walk_out.keep, walk_out.accepted, pk, pv)
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
    rec = {"what": args.what, "config": args.config, "batch": w.B,
           "us_per_launch": round(ev[0].elapsed_time(ev[1]) * 1e3 / args.iters, 1)}
    if args.graph:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            once()
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(args.iters):
                once()
        graph.replay()
        torch.cuda.synchronize()
        ev[0].record()
        graph.replay()
        ev[1].record()
        torch.cuda.synchronize()
        if _lib.device_error() != 0:
            raise RuntimeError("device error")
        rec["us_per_launch_graph"] = round(ev[0].elapsed_time(ev[1]) * 1e3 / args.iters, 1)
    if args.what in ("attn", "attn_store"):
        # achieved work against the measured peaks (MEASURED_PEAKS.json beside the package, else the
        # earlier measurement on this pool); a kernel timed alone is compared with the burst figures
        import pathlib
        cnt = trees.count.cpu().tolist()
        dep = trees.depth.cpu()
        depth_sums = [int(dep[b, :cnt[b]].sum()) for b in range(w.B)]
        flops, nbytes = w.attn_flops(depth_sums), w.attn_bytes()
        t_s = rec["us_per_launch"] * 1e-6
        peaks = pathlib.Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"
        if peaks.exists():
            pk = json.loads(peaks.read_text())
            hbm, tf, src = float(pk["hbm_gbs"]), float(pk["bf16_tflops"]), "measured"
        else:
            hbm, tf, src = 6650.0, 1590.0, "fallback"
        rec["tflops"] = round(flops / t_s / 1e12, 1)
        rec["gbs"] = round(nbytes / t_s / 1e9, 1)
        rec["hbm_floor_us"] = round(nbytes / (hbm * 1e9) * 1e6, 1)
        if dtype != torch.float32:
            rec["tensor_floor_us"] = round(flops / (tf * 1e12) * 1e6, 1)
            bound = "tensor" if rec["tensor_floor_us"] >= rec["hbm_floor_us"] else "hbm"
            rec["bound"] = bound
            rec["frac_of_burst_peak"] = round((rec["tflops"] / tf) if bound == "tensor" else (rec["gbs"] / hbm), 3)
        rec["peaks"] = src
        if args.what == "attn":
            kern, n_split, _ = cast_b200.attention_plan(q, k, v, out, w.B, lay["max_pack"], lay["max_kv"])
            # the library's dispatch (capi.cu): pairs when the largest head group fills whole 256-row
            # pairs; pairs for the full blocks and single CTAs for the last ones when it is longer than a
            # pair, ends in a one-tile block and the key chunks hold 64 tiles or more; else single CTAs
            gmp = (w.H_q // w.H_kv) * lay["max_pack"]
            chunk_tiles = -(-lay["max_kv"] // n_split // 128)
            auto = kern == "tcgen05" and args.kernel == "auto"
            if auto and gmp % 256 == 0:
                rec["kernel"] = "tcgen05 CTA pairs"
            elif auto and gmp > 256 and gmp % 256 <= 128 and chunk_tiles >= 64:
                rec["kernel"] = "tcgen05 CTA pairs (full blocks) + single CTAs (last blocks)"
            else:
                rec["kernel"] = "tcgen05 single CTAs" if kern == "tcgen05" else kern
            rec["key_splits"] = n_split
    if args.what in ("walk", "append"):
        acc = walk_out.accepted.cpu()
        rec["mean_accepted"] = round(float(acc.float().mean()), 2)
        rec["max_accepted"] = int(acc.max())
        rec["rows_read"] = int(acc.sum())    # logits rows the walk read: one per accepted token
    print(json.dumps(rec))


if __name__ == "__main__":
    main()
