"""Benchmark of the ragged tree-verification hot path on B200.

One step = one verify round over a batch, as CAST runs it: GPU block_topk of
the drafter's fp64 block scores and GPU best-first tree build (pack parents
written in the same launch) once per round, then one ragged tree-attention
call per decoder layer consuming those parents (cast_trees/serving.py calls
its attention hook once per layer of the target forward). Workload at N=1:
BASELINE configuration 3 (B=64, N=127, prefix ~ U[4096,8192], Llama-3.1-8B
attention geometry 32/8 heads, d=128, 32 layers, bf16, V=128256), synthetic;
the layers share one synthetic K/V set (1.59 GB, far larger than L2, so each
call streams it from HBM).
With --gpus N (one process per GPU under torchrun) every rank runs its own
64 sequences of the same recipe (weak scaling, no collective on the path).

Prints one JSON line (rank 0). `value` is attention TFLOP/s of the whole job
(visible (query, key) pairs only, 4 flops per pair and dim) over the device
time of the full step; `e2e` is the same metric through the public Python API
with pinned host inputs copied in and the output copied out inside the timed
region. `--impl reference` times the reference's CPU path (the oracle port of
cast_trees' numpy block_topk/build_tree and the fp32 masked-softmax reference
of tests/test_tree_attn.py) on the host cores.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "tree-attn µs/call and TFLOP/s, B=64 N=127 ctx 4-8K; % of roofline at 1-8 GPUs"
B_PER_RANK = 64
N_NODES = 127


def _env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d["bf16_tflops_sustained"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def _profile_traffic(name):
    """dram bytes per launch from a committed ncu summary line 'traffic_bytes_per_launch[<name>]: X'."""
    for f in sorted((ROOT / "profiles").glob("*.md")):
        for line in f.read_text().splitlines():
            key = f"traffic_bytes_per_launch[{name}]:"
            if line.strip().startswith(key):
                try:
                    return float(line.split(":", 1)[1].strip().split()[0])
                except ValueError:
                    return None
    return None


class ClockSampler:
    """nvidia-smi clock / throttle samples during the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = []
        try:
            for line in Path(self.path).read_text().splitlines():
                f = [x.strip() for x in line.split(",")]
                if len(f) >= 9 and f[1].replace(".", "").isdigit():
                    rows.append(f)
        except OSError:
            pass
        finally:
            try:
                os.unlink(self.path)
            except OSError:
                pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows)}


def rank_workload(rank):
    from cast_b200 import workloads
    full = workloads.Workload("config3", 2, 128256, *workloads._ragged(2, B_PER_RANK * (rank + 1), 4096, 8192, (N_NODES,)))
    return full.shard(list(range(rank * B_PER_RANK, (rank + 1) * B_PER_RANK)))


class Step:
    """Device buffers and the three launches of one verify pass."""

    def __init__(self, w, dev):
        import cast_b200
        self.cb = cast_b200
        self.w = w
        self.dev = dev
        lay = w.layout()
        self.lay = lay
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        self.cu_q, self.cu_kv = t(lay["cu_q"]), t(lay["cu_kv"])
        self.prefix, self.pack = t(lay["prefix_len"]), t(lay["pack_len"])
        self.budget = torch.full((w.B,), N_NODES, dtype=torch.int32, device=dev)
        self.roots = torch.zeros(w.B, dtype=torch.int32, device=dev)
        self.seq_len = self.prefix.clone()
        self.logits = torch.empty((w.B, 15, w.V), dtype=torch.float64, device=dev)
        self.q = self.k = self.v = None
        self.out = None
        self.idx = torch.empty((w.B, 15, 8), dtype=torch.int64, device=dev)
        self.lp = torch.empty((w.B, 15, 8), dtype=torch.float64, device=dev)
        self.ws = None

    def run(self, layers, ev=None):
        """One verify round; ev: optional (start, end) events around the attention calls."""
        cb = self.cb
        cb.block_topk_device(self.logits, 8, self.idx, self.lp)
        trees = cb.build_trees(self.idx, self.lp, self.budget, 8, max_budget=N_NODES, cu_q=self.cu_q,
                               root_token=self.roots, seq_len=self.seq_len, total_q=self.lay["total_q"])
        if ev is not None:
            ev[0].record()
        for _ in range(layers):
            self.out = cb.varlen_tree_attention(self.q, self.k, self.v, self.cu_q, self.cu_kv, self.prefix,
                                                self.pack, None, parent=trees.pack_parent,
                                                max_pack=self.lay["max_pack"], max_kv=self.lay["max_kv"],
                                                out=self.out, workspace=self.ws)
        if ev is not None:
            ev[1].record()
        return trees


def run_cast(args):
    import torch.distributed as dist
    rank, world, local = _env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    import cast_b200
    from cast_b200 import _lib

    w = rank_workload(rank)
    st = Step(w, dev)
    # host inputs (pinned): the e2e leg copies them every step
    h_logits = torch.empty((w.B, 15, w.V), dtype=torch.float64).pin_memory()
    w.logits_batch(out=h_logits)
    st.logits.copy_(h_logits)
    st.q, st.k, st.v = w.make_qkv(dev)
    h_q, h_k, h_v = (x.cpu().pin_memory() for x in (st.q, st.k, st.v))
    st.out = torch.empty_like(st.q)
    h_out = torch.empty(st.out.shape, dtype=st.out.dtype).pin_memory()
    ws = cast_b200.workspace_size(w.dtype, w.B, w.layout()["total_q"], w.H_q, w.H_kv, w.D,
                                  w.layout()["max_pack"], w.layout()["max_kv"])
    st.ws = torch.empty(max(ws, 1), dtype=torch.uint8, device=dev)

    # launches per step: block_topk + build_tree + attention (+ combine when the keys are split)
    kernel, n_split, attn_launches = cast_b200.attention_plan(st.q, st.k, st.v, st.out, w.B, w.layout()["max_pack"],
                                                              w.layout()["max_kv"])
    launches_per_step = 3 + attn_launches * args.layers   # topk (fast + exact kernels), tree, attention

    for _ in range(args.warmup):
        trees = st.run(args.layers)
    torch.cuda.synchronize()
    err = _lib.device_error()
    if err != 0:
        raise RuntimeError(f"device error {err} after warm-up")
    depth_sums = trees.depth.sum(dim=1, dtype=torch.int64).cpu().tolist()
    call_flops = w.attn_flops(depth_sums)
    call_bytes = w.attn_bytes()
    flops = call_flops * args.layers          # per step

    stream = torch.cuda.current_stream()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = ClockSampler(local).__enter__()      # sampled over both timed regions below
    time.sleep(0.3)                            # nvidia-smi start-up
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0.record(stream)
    for i in range(args.steps):
        st.run(args.layers, evs[i])
    t1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    step_ms = t0.elapsed_time(t1) / args.steps
    attn_ms = statistics.mean(a.elapsed_time(b) for a, b in evs) / args.layers   # per call
    tree_ms = step_ms - attn_ms * args.layers

    # e2e: the public API with host buffers, every step's copies inside the timed region. The
    # loop is pipelined the way a server runs it: two device input sets, the host-to-device
    # copies of step i+1 on a copy stream while step i computes, each result read back on a
    # third stream (both copy directions overlap the compute).
    h2d = sum(x.numel() * x.element_size() for x in (h_logits, h_q, h_k, h_v))
    d2h = h_out.numel() * h_out.element_size()
    names = ("logits", "q", "k", "v")
    hosts = dict(logits=h_logits, q=h_q, k=h_k, v=h_v)
    bufs = [dict(logits=st.logits, q=st.q, k=st.k, v=st.v, out=st.out),
            dict(logits=torch.empty_like(st.logits), q=torch.empty_like(st.q), k=torch.empty_like(st.k),
                 v=torch.empty_like(st.v), out=torch.empty_like(st.out))]
    h2d_stream, d2h_stream = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    copied = [torch.cuda.Event(), torch.cuda.Event()]     # inputs of set b are on the device
    used = [torch.cuda.Event(), torch.cuda.Event()]       # the step on set b has read its inputs
    read = [torch.cuda.Event(), torch.cuda.Event()]       # the result of set b is on the host

    def issue_copy(b):
        h2d_stream.wait_event(used[b])
        with torch.cuda.stream(h2d_stream):
            for n in names:
                bufs[b][n].copy_(hosts[n], non_blocking=True)
        copied[b].record(h2d_stream)

    def e2e_steps(n):
        h2d_stream.wait_stream(stream)
        d2h_stream.wait_stream(stream)
        issue_copy(0)
        for i in range(n):
            b = i % 2
            if i + 1 < n:
                issue_copy(1 - b)
            stream.wait_event(copied[b])
            stream.wait_event(read[b])
            st.logits, st.q, st.k, st.v, st.out = (bufs[b][x] for x in ("logits", "q", "k", "v", "out"))
            st.run(args.layers)
            used[b].record(stream)
            d2h_stream.wait_event(used[b])
            with torch.cuda.stream(d2h_stream):
                h_out.copy_(bufs[b]["out"], non_blocking=True)
            read[b].record(d2h_stream)
        stream.wait_stream(h2d_stream)
        stream.wait_stream(d2h_stream)

    e2e_steps(max(1, args.warmup))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    e2e_steps(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    clk.__exit__(None, None, None)
    if world > 1:
        dist.barrier()
    e2e_ms = e0.elapsed_time(e1) / args.steps

    # max over ranks of every time; sums of work
    t = torch.tensor([step_ms, attn_ms, tree_ms, e2e_ms], dtype=torch.float64, device=dev)
    work = torch.tensor([flops, call_bytes], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(work, op=dist.ReduceOp.SUM)
    step_ms, attn_ms, tree_ms, e2e_ms = t.tolist()
    tot_flops, tot_bytes = work.tolist()
    hbm, tf_burst, tf_sus, peak_kind = _peaks()

    value = tot_flops / (step_ms * 1e-3) / 1e12
    attn_tflops = call_flops / (attn_ms * 1e-3) / 1e12     # per GPU, dominant kernel, per call
    attn_gbs = call_bytes / (attn_ms * 1e-3) / 1e9
    topk_gbs = w.topk_bytes() / (tree_ms * 1e-3) / 1e9
    # binding roofline of the attention kernel: the slower of the HBM and tensor floors. The
    # kernel runs `layers` times back to back inside a long step (power-capped clocks), so the
    # tensor peak is the sustained figure; the burst figure is reported beside it.
    tf_peak = tf_sus
    t_hbm = call_bytes / (hbm * 1e9)
    t_tensor = call_flops / (tf_peak * 1e12)
    bound = "tensor" if t_tensor >= t_hbm else "hbm"
    if bound == "tensor":
        roof = {"bound": "tensor", "achieved": round(attn_tflops, 2), "peak": tf_peak, "unit": "TFLOP/s",
                "frac": round(attn_tflops / tf_peak, 4)}
    else:
        roof = {"bound": "hbm", "achieved": round(attn_gbs, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(attn_gbs / hbm, 4)}
    roof["traffic"] = _profile_traffic("attn_config3")
    roof["peak_source"] = (f"{peak_kind}: MEASURED_PEAKS.json bf16_tflops_sustained (kernel timed inside a long "
                           f"step); hbm_gbs for the HBM floor")
    roof["frac_of_burst_peak"] = round(attn_tflops / tf_burst, 4)
    roof["hbm_floor_us"] = round(t_hbm * 1e6, 1)
    roof["tensor_floor_us"] = round(t_tensor * 1e6, 1)

    result = {
        "metric": METRIC, "value": round(value, 3), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded normal(scale=5) block scores 15x128256 fp64, q/k/v N(0,1)*0.5 bf16",
        "config": {"workload": f"config3: B=64/GPU, N=127 (P=128), prefix U[4096,8192], 32/8 heads, d=128, "
                               f"V=128256; step = one verify round: block_topk + build_tree + {args.layers} "
                               f"tree-attention calls (one per layer)", "layers": args.layers,
                   "global_batch": B_PER_RANK * world, "seq_len": "4096-8192 (ragged)",
                   "parallelism": f"sequence-sharded x{world}, no collective",
                   "l2": "inputs larger than L2 (logits 0.98 GB + K/V 1.59 GB streamed per step)"},
        "attn_kernel": kernel, "attn_key_splits": n_split,
        "us_per_call": round(attn_ms * 1e3, 1),
        "attn_tflops_per_gpu": round(attn_tflops, 2),
        "attn_gbs_per_gpu": round(attn_gbs, 1),
        "tree_build_us": round(tree_ms * 1e3, 1),
        "tree_build_gbs": round(topk_gbs, 1),
        "roofline": roof,
        "e2e": {"value": round(tot_flops / (e2e_ms * 1e-3) / 1e12, 4), "unit": "TFLOP/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 3),
                "pipelined": "two device input sets; step i+1's host-to-device copies and step i's result "
                             "read overlap step i's compute"},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk.summary(),
    }
    result["verify_round_rows"] = round_rows(st, trees, w, dev)
    if world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(w, trees, args)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        emit(result)


def round_rows(st, trees, w, dev, iters=10):
    """Per-call device time of the verify-round steps after attention, on this rank's batch.

    walk: greedy walk over synthetic bf16 target logits [total_q, V] that follow each tree's
    first child with probability 3/4; select: select_global_topk_device keeping 48 nodes per
    request; append: the walk's accepted rows into 32 layers of per-request stores in place
    (the kernel's work depends only on the appended rows, so the stores hold no prefix here).
    CUDA events around `iters` eager calls each.
    """
    try:
        import cast_b200
        lay = st.lay
        gen = torch.Generator(device=dev).manual_seed(7)
        V = w.V
        tl = torch.empty((lay["total_q"], V), dtype=torch.bfloat16, device=dev)
        tl.normal_(generator=gen)
        pp = trees.pack_parent
        ptok = torch.where(pp >= 0, torch.randint(0, V, pp.shape, device=dev, dtype=torch.int32, generator=gen),
                           torch.zeros_like(pp))
        rows = torch.arange(lay["total_q"], device=dev)
        q0 = torch.repeat_interleave(st.cu_q[:-1].long(), st.pack.long())
        par_abs = torch.where(pp >= 0, q0 + pp.long(), torch.full_like(q0, -1))
        big = torch.iinfo(torch.int64).max
        first = torch.full((lay["total_q"],), big, dtype=torch.int64, device=dev)
        child = rows[par_abs >= 0]
        first.scatter_reduce_(0, par_abs[child], child, reduce="amin")
        has = (first < big) & (torch.rand(first.shape, generator=gen, device=dev) < 0.75)
        tl[rows[has], ptok[first[has]].long()] = 50.0
        cap = lay["max_pack"] - 1
        walk = cast_b200.walk_trees_greedy(tl, st.cu_q, pp, ptok, cap)
        n_layers = 32
        mk = lambda: torch.zeros((w.B, w.H_kv, 32, w.D), dtype=torch.bfloat16, device=dev)
        bk, bv = [mk() for _ in range(n_layers)], [mk() for _ in range(n_layers)]
        pk = [torch.randn((w.H_kv, lay["total_q"], w.D), device=dev).to(torch.bfloat16) for _ in range(n_layers)]
        pv = [torch.randn((w.H_kv, lay["total_q"], w.D), device=dev).to(torch.bfloat16) for _ in range(n_layers)]
        zero = torch.zeros(w.B, dtype=torch.int32, device=dev)

        def timed(fn):
            fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(iters):
                fn()
            e1.record()
            torch.cuda.synchronize()
            return round(e0.elapsed_time(e1) * 1e3 / iters, 1)

        res = {
            "walk_us": timed(lambda: cast_b200.walk_trees_greedy(tl, st.cu_q, pp, ptok, cap, out=walk)),
            "select_us": timed(lambda: cast_b200.select_global_topk_device(trees, 48 * w.B,
                                                                           pack_capacity=49 * w.B)),
            "append_us": timed(lambda: cast_b200.append_store_inplace(bk, bv, zero, st.cu_q[:-1], walk.keep,
                                                                      walk.accepted, pk, pv)),
        }
        acc = walk.accepted.float()
        res["mean_accepted"] = round(float(acc.mean()), 2)
        res["rows_walked"] = int(acc.sum())
        res["note"] = (f"{w.B} requests, V={V} bf16 target logits, select keeps 48 of {trees.token.shape[1]} "
                       f"nodes per request, append covers {n_layers} layers x K,V; eager calls (host time "
                       f"included), device-only times in profiles/")
        from cast_b200 import _lib
        if _lib.device_error() != 0:
            res["error"] = "device error"
        return res
    except Exception as e:   # the round's steps are reported beside the metric, never instead of it
        return {"error": f"{type(e).__name__}: {e}"}


def _cpu_sample(w, ids):
    """Times the oracle (the reference's CPU algorithms) on sequences `ids` of w.

    Returns (tree_seconds, attention_seconds_per_call, flops_per_call, trees):
    numpy block_topk + heap build_tree once, then one fp32 masked-softmax
    attention call (torch, all threads). q/k/v are drawn on the CPU.
    """
    from oracle import attn as oattn
    from oracle import tree as otree
    sub = w.shard(ids)
    lay = sub.layout()
    g = torch.Generator().manual_seed(1234)
    q = (torch.randn(lay["total_q"], w.H_q, w.D, generator=g) * 0.5).to(w.dtype)
    k = (torch.randn(lay["total_kv"], w.H_kv, w.D, generator=g) * 0.5).to(w.dtype)
    v = (torch.randn(lay["total_kv"], w.H_kv, w.D, generator=g) * 0.5).to(w.dtype)
    logits = [sub.logits(b) for b in range(sub.B)]
    t0 = time.perf_counter()
    trees, words = [], []
    for b in range(sub.B):
        idx, lp = otree.block_topk(logits[b])
        tr = otree.build_tree(idx, lp, sub.N[b])
        trees.append(tr)
        words.append(otree.ancestor_words(otree.pack_parent(tr.parent)))
    t1 = time.perf_counter()
    oattn.tree_attention(q.float(), k.float(), v.float(), lay["cu_q"], lay["cu_kv"], lay["prefix_len"],
                         lay["pack_len"], words)
    t2 = time.perf_counter()
    flops = sub.attn_flops([int(t.depth.sum()) for t in trees])
    return t1 - t0, t2 - t1, flops, trees


def cpu_baseline(w, trees_gpu, args):
    n = max(1, args.cpu_seqs)
    torch.set_num_threads(os.cpu_count() or 1)
    t_tree, t_attn, flops, trees = _cpu_sample(w, list(range(n)))
    round_s = t_tree + args.layers * t_attn
    exact = True
    for b in range(n):
        c = int(trees_gpu.count[b])
        exact &= c == len(trees[b])
        exact &= np.array_equal(trees_gpu.parent[b, :c].cpu().numpy(), trees[b].parent)
        exact &= np.array_equal(trees_gpu.token[b, :c].cpu().numpy(), trees[b].token)
        exact &= np.array_equal(trees_gpu.depth[b, :c].cpu().numpy(), trees[b].depth)
    return {"value": round(args.layers * flops / round_s / 1e12, 6), "unit": "TFLOP/s",
            "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{n} of the {w.B} config-3 sequences: numpy block_topk + heap build_tree once "
                      f"({t_tree:.2f} s, 1 thread) and one fp32 masked-softmax attention call "
                      f"({t_attn:.3f} s, torch, all threads) counted {args.layers}x (one per layer)",
            "tree_arrays_bit_exact_vs_gpu": bool(exact)}


def run_reference(args):
    rank, world, local = _env()
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    w = rank_workload(0)
    n = max(1, args.ref_seqs)
    times, flops = [], 0
    for i in range(args.warmup + args.steps):
        ids = [(i * n + j) % w.B for j in range(n)]
        t_tree, t_attn, fl, _ = _cpu_sample(w, ids)
        if i >= args.warmup:
            times.append(t_tree + args.layers * t_attn)
            flops += fl * args.layers
    tot = sum(times)
    value = flops / tot / 1e12
    emit({
        "metric": METRIC, "impl": "reference", "value": round(value, 6), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * tot / args.steps, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16 inputs, fp32 compute",
        "data": "synthetic (config-3 recipe)",
        "config": {"workload": f"config3 sample: {n} sequences per step, one verify round (block_topk + "
                               f"build_tree once, attention counted once per layer, {args.layers} layers)",
                   "global_batch": n, "seq_len": "4096-8192 (ragged)", "parallelism": "host CPU",
                   "layers": args.layers},
        "cpu_baseline": {"value": round(value, 6), "unit": "TFLOP/s", "cores": torch.get_num_threads(),
                         "kind": "port", "sample": f"{n} config-3 sequences per step; the reference is Python: "
                                                   f"its numpy tree builder and its fp32 masked-softmax attention"},
        "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    })


_JSON_FD = None


def emit(obj):
    """The one JSON line, on the real stdout (fd 1 itself is pointed at stderr in main())."""
    os.write(_JSON_FD if _JSON_FD is not None else 1, (json.dumps(obj) + "\n").encode())


def main():
    global _JSON_FD
    # whatever the libraries print on stdout (NCCL's version line, for one) goes to stderr;
    # stdout carries only the JSON line
    sys.stdout.flush()
    _JSON_FD = os.dup(1)
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["cast", "reference"], default="cast")
    ap.add_argument("--layers", type=int, default=32, help="attention calls per verify round (decoder layers)")
    ap.add_argument("--cpu-seqs", type=int, default=8, help="sequences in the cpu_baseline sample")
    ap.add_argument("--ref-seqs", type=int, default=2, help="sequences per step of --impl reference")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_cast(args)


if __name__ == "__main__":
    main()
