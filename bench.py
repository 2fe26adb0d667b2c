"""Benchmark of the ragged tree-verification hot path on B200.

One step = one verify round over a batch, as CAST runs it: GPU block_topk of
the drafter's fp64 block scores and GPU best-first tree build (pack parents
written in the same launch) once per round, then one ragged tree-attention
call per decoder layer consuming those parents (cast_trees/serving.py calls
its attention hook once per layer of the target forward). Workload at N=1:
configuration 3 of cast_b200.workloads (B=64, N=127, prefix ~ U[4096,8192],
Llama-3.1-8B attention geometry 32/8 heads, d=128, 32 layers, bf16,
V=128256), synthetic; the layers share one synthetic K/V set (1.59 GB, far
larger than L2, so each call streams it from HBM).

With --gpus N (one process per GPU under torchrun) the job draws one batch of
64 * N sequences of the same recipe (the first 64 are configuration 3) and
splits it into equal-count shards of near-equal cost, 64 sequences per rank
(weak scaling, no collective on the path); times are the max over ranks.

Prints one JSON line (rank 0). `value` is attention TFLOP/s of the whole job
(visible (query, key) pairs only, 4 flops per pair and dim) over the device
time of the full step; `e2e` is the same metric through the public Python API
with pinned host inputs copied in and the output copied out inside the timed
region. Beside the metric, measured outside the timed regions:
  roofline   the attention kernel against the measured burst bf16 peak (the
             kernel runs at full clocks inside the round); DRAM traffic per
             launch only when --traffic-csv names an ncu capture of it
  parity     max abs error of the timed attention output against the CPU
             oracle on a seeded sample of sequences
  config5    configuration 5: one fixed batch of 512 sequences sharded by cost
             over the N GPUs (strong scaling), one attention call per tree
             width N in {16..256}: l(N) (max over ranks), fraction of the
             binding roofline, and the least-squares c0/c1 over 16 <= n <= 128
             fed to cast_trees.width.predict_width when the reference package
             is installed beside the repo (baseline/_ref)
  cpu_baseline  (N=1) the oracle port of the reference's CPU path timed on a
             sample of the same round on the host cores
`--impl reference` times that CPU path (the reference's numpy tree builder and
its fp32 masked-softmax attention, restated in oracle/) one sampled sequence
per step, full round per step, and prints the same line with impl=reference.
The CPU legs (cpu_baseline, parity, the reference arm) are the only users of
oracle/, always outside the timed regions.
"""
import argparse
import csv
import json
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
LAYERS_DEFAULT = 32
TOL_BF16 = 2e-2
WIDTHS = (16, 24, 32, 48, 64, 96, 128, 256)


def _env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d["bf16_tflops_sustained"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def _traffic_from_csv(path, kernel="attn_tc_kernel"):
    """dram read + write bytes per launch of `kernel` from an ncu --csv capture (raw or details page)."""
    vals = {}
    with open(path, newline="") as f:
        rows = [r for r in csv.reader(f) if r]
    head = next((i for i, r in enumerate(rows) if "Kernel Name" in r), None)
    if head is None:
        return None
    cols = rows[head]
    kn = cols.index("Kernel Name")
    if "Metric Name" in cols:   # details page: one row per metric
        mn, mv, mu = cols.index("Metric Name"), cols.index("Metric Value"), cols.index("Metric Unit")
        scale = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9}
        for r in rows[head + 1:]:
            if kernel in r[kn] and r[mn] in ("dram__bytes_read.sum", "dram__bytes_write.sum"):
                vals.setdefault(r[mn], []).append(float(r[mv].replace(",", "")) * scale.get(r[mu], 1))
    else:                       # raw page: one row per launch, one column per metric (units in the next row)
        units = rows[head + 1]
        for name in ("dram__bytes_read.sum", "dram__bytes_write.sum"):
            if name in cols:
                c = cols.index(name)
                sc = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9}.get(units[c], 1)
                vals[name] = [float(r[c].replace(",", "")) * sc for r in rows[head + 2:] if kernel in r[kn]]
    if len(vals) != 2 or not all(vals.values()):
        return None
    n = min(len(v) for v in vals.values())
    return sum(sum(v[:n]) for v in vals.values()) / n


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


def job_workload(world):
    """The whole job's batch: 64 * world sequences of the configuration-3 recipe (seed 2)."""
    from cast_b200 import workloads
    S, N = workloads._ragged(2, B_PER_RANK * world, 4096, 8192, (N_NODES,))
    return workloads.Workload("config3", 2, 128256, S, N)


def rank_workload(rank, world):
    """This rank's 64 sequences: equal-count shards of near-equal attention cost."""
    from cast_b200 import sharding
    full = job_workload(world)
    costs = [sharding.sequence_cost(s, p) for s, p in zip(full.S, full.P)]
    return full.shard(sharding.equal_count_shards(costs, world, B_PER_RANK)[rank])


def bench_config(args, world):
    """The `config` object of the JSON line (identical for both arms)."""
    return {"workload": f"config3: B=64/GPU, N=127 (P=128), prefix U[4096,8192], 32/8 heads, d=128, V=128256; "
                        f"step = one verify round: block_topk + build_tree + {args.layers} tree-attention calls "
                        f"(one per layer)",
            "layers": args.layers, "global_batch": B_PER_RANK * world, "seq_len": "4096-8192 (ragged)",
            "parallelism": f"sequence-sharded x{world} (equal-count cost-balanced shards), no collective",
            "l2": "inputs larger than L2 (logits 0.98 GB + K/V 1.59 GB streamed per step)"}


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
        """One verify round; ev: optional (start, end, tree start) events: the first two around the
        attention calls, the third before the tree build."""
        cb = self.cb
        if ev is not None and len(ev) > 2:
            ev[2].record()
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


def _dist():
    import torch.distributed as dist
    return dist


def _max_over_ranks(vals, dev, world, op="max"):
    t = torch.tensor(vals, dtype=torch.float64, device=dev)
    if world > 1:
        dist = _dist()
        dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return t.tolist()


def run_cast(args):
    rank, world, local = _env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        _dist().init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    import cast_b200
    from cast_b200 import _lib

    w = rank_workload(rank, world)
    st = Step(w, dev)
    # host inputs (pinned): the e2e leg copies them every step
    h_logits = torch.empty((w.B, 15, w.V), dtype=torch.float64).pin_memory()
    w.logits_batch(out=h_logits)
    st.logits.copy_(h_logits)
    st.q, st.k, st.v = w.make_qkv(dev)
    h_q, h_k, h_v = (x.cpu().pin_memory() for x in (st.q, st.k, st.v))
    st.out = torch.empty_like(st.q)
    h_out = torch.empty(st.out.shape, dtype=st.out.dtype).pin_memory()
    lay = w.layout()
    ws = cast_b200.workspace_size(w.dtype, w.B, lay["total_q"], w.H_q, w.H_kv, w.D, lay["max_pack"], lay["max_kv"])
    st.ws = torch.empty(max(ws, 1), dtype=torch.uint8, device=dev)

    # launches per step: block_topk (fast + exact kernels) + build_tree + attention (+ combine when split)
    kernel, n_split, attn_launches = cast_b200.attention_plan(st.q, st.k, st.v, st.out, w.B, lay["max_pack"],
                                                              lay["max_kv"])
    launches_per_step = 3 + attn_launches * args.layers

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
    evs = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(3)) for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = ClockSampler(local).__enter__()      # sampled over both timed regions below
    time.sleep(0.3)                            # nvidia-smi start-up
    if world > 1:
        _dist().barrier()
    torch.cuda.synchronize()
    t0.record(stream)
    for i in range(args.steps):
        st.run(args.layers, evs[i])
    t1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        _dist().barrier()
    step_ms = t0.elapsed_time(t1) / args.steps
    attn_ms = statistics.mean(a.elapsed_time(b) for a, b, _ in evs) / args.layers   # per call
    tree_ms = statistics.mean(t.elapsed_time(a) for a, _, t in evs)                  # block_topk + build_tree

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
        _dist().barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    e2e_steps(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    clk.__exit__(None, None, None)
    if world > 1:
        _dist().barrier()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if _lib.device_error() != 0:
        raise RuntimeError("device error in the timed regions")

    # max over ranks of every time; sums of work
    step_ms, attn_ms, tree_ms, e2e_ms = _max_over_ranks([step_ms, attn_ms, tree_ms, e2e_ms], dev, world)
    tot_flops, tot_bytes = _max_over_ranks([flops, call_bytes], dev, world, op="sum")
    hbm, tf_burst, tf_sus, peak_kind = _peaks()

    value = tot_flops / (step_ms * 1e-3) / 1e12
    attn_tflops = call_flops / (attn_ms * 1e-3) / 1e12     # per GPU, dominant kernel, per call
    attn_gbs = call_bytes / (attn_ms * 1e-3) / 1e9
    topk_gbs = w.topk_bytes() / (tree_ms * 1e-3) / 1e9
    # binding roofline of the attention kernel: the slower of the HBM and tensor floors, against
    # the burst peaks (the kernel's clocks stay near the maximum inside the round: see `clocks`)
    t_hbm = call_bytes / (hbm * 1e9)
    t_tensor = call_flops / (tf_burst * 1e12)
    bound = "tensor" if t_tensor >= t_hbm else "hbm"
    if bound == "tensor":
        roof = {"bound": "tensor", "achieved": round(attn_tflops, 2), "peak": tf_burst, "unit": "TFLOP/s",
                "frac": round(attn_tflops / tf_burst, 4)}
    else:
        roof = {"bound": "hbm", "achieved": round(attn_gbs, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(attn_gbs / hbm, 4)}
    roof["traffic"] = _traffic_from_csv(args.traffic_csv) if args.traffic_csv else None
    if roof["traffic"] is not None:
        roof["traffic_over_algorithmic"] = round(roof["traffic"] / call_bytes, 3)
        roof["traffic_source"] = f"ncu capture {args.traffic_csv}"
    roof["peak_source"] = (f"{peak_kind}: MEASURED_PEAKS.json bf16_tflops (burst) for the tensor floor, hbm_gbs "
                           f"for the HBM floor; achieved = algorithmic flops per call / CUDA-event time per call")
    roof["frac_of_sustained_peak"] = round(attn_tflops / tf_sus, 4)
    roof["algorithmic_flops_per_call"] = call_flops
    roof["algorithmic_bytes_per_call"] = call_bytes
    roof["hbm_floor_us"] = round(t_hbm * 1e6, 1)
    roof["tensor_floor_us"] = round(t_tensor * 1e6, 1)

    result = {
        "metric": METRIC, "value": round(value, 3), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded normal(scale=5) block scores 15x128256 fp64, q/k/v N(0,1)*0.5 bf16",
        "config": bench_config(args, world),
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
    # CPU legs (oracle), outside every timed region
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(w, st, trees, args)
        result["cpu_baseline"] = cpu["baseline"]
    result["parity"] = parity_check(w, st, trees, dev, world, rank, cpu)
    if not args.no_config5:
        result["config5"] = config5_sweep(dev, world, rank, hbm, tf_burst, args)
    if world > 1:
        _dist().barrier()
        _dist().destroy_process_group()
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
                       f"nodes per request, append covers {n_layers} layers x K,V; eager calls, host time included")
        from cast_b200 import _lib
        if _lib.device_error() != 0:
            res["error"] = "device error"
        return res
    except Exception as e:   # the round's steps are reported beside the metric, never instead of it
        return {"error": f"{type(e).__name__}: {e}"}


def _seq_inputs(w, st, b):
    """CPU copies of sequence b's q, k, v rows (the bench's own device inputs)."""
    lay = w.layout()
    cq, ckv = lay["cu_q"], lay["cu_kv"]
    return (st.q[cq[b]:cq[b + 1]].cpu(), st.k[ckv[b]:ckv[b + 1]].cpu(), st.v[ckv[b]:ckv[b + 1]].cpu())


def _cpu_round(w, b, layers, qkv):
    """The reference's CPU path for one sequence of the round, timed (oracle port).

    numpy block_topk + heap build_tree (cast_trees/tree.py:20-49, single-threaded as in the
    reference), then `layers` fp32 masked-softmax attention calls (tests/test_tree_attn.py:40-59,
    torch with all threads). Returns (tree_s, attn_s, flops, tree, out).
    """
    from oracle import attn as oattn
    from oracle import tree as otree
    logits = w.logits(b)
    t0 = time.perf_counter()
    idx, lp = otree.block_topk(logits)
    tr = otree.build_tree(idx, lp, w.N[b])
    words = [otree.ancestor_words(otree.pack_parent(tr.parent))]
    t1 = time.perf_counter()
    q, k, v = (x.float() for x in qkv)
    S, P = w.S[b], w.P[b]
    out = None
    for _ in range(layers):
        out = oattn.tree_attention(q, k, v, [0, P], [0, S + P], [S], [P], words)
    t2 = time.perf_counter()
    flops = layers * 4 * w.H_q * w.D * (P * S + P + int(tr.depth.sum()))
    return t1 - t0, t2 - t1, flops, tr, out


def cpu_baseline(w, st, trees_gpu, args):
    """Oracle port of the reference's CPU path on a sample of this round (rank 0, N=1)."""
    torch.set_num_threads(os.cpu_count() or 1)
    ids = list(range(max(1, args.cpu_seqs)))
    t_tree = t_attn = 0.0
    flops = 0
    exact = True
    outs = {}
    for b in ids:
        tt, ta, fl, tr, out = _cpu_round(w, b, args.layers, _seq_inputs(w, st, b))
        t_tree += tt
        t_attn += ta
        flops += fl
        outs[b] = out
        c = int(trees_gpu.count[b])
        exact &= c == len(tr)
        exact &= np.array_equal(trees_gpu.parent[b, :c].cpu().numpy(), tr.parent)
        exact &= np.array_equal(trees_gpu.token[b, :c].cpu().numpy(), tr.token)
        exact &= np.array_equal(trees_gpu.depth[b, :c].cpu().numpy(), tr.depth)
    base = {"value": round(flops / (t_tree + t_attn) / 1e12, 6), "unit": "TFLOP/s",
            "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{len(ids)} of the {w.B} sequences of this round, each a full round: numpy block_topk + "
                      f"heap build_tree ({t_tree:.2f} s in all, 1 thread) and {args.layers} fp32 masked-softmax "
                      f"attention calls ({t_attn:.2f} s in all, torch, all threads); measured, not projected",
            "tree_arrays_bit_exact_vs_gpu": bool(exact)}
    return {"baseline": base, "outs": outs}


def parity_check(w, st, trees, dev, world, rank, cpu=None):
    """Max abs error of the timed attention output against the oracle on sampled sequences.

    The output checked is the last timed call's (every layer reads the same inputs); the oracle
    runs on the same bf16 inputs and on the GPU-built tree. Max over ranks.
    """
    from oracle import attn as oattn
    from oracle import tree as otree
    lay = w.layout()
    cq = lay["cu_q"]
    if cpu is not None:
        outs = cpu["outs"]
    else:
        outs = {}
        pp = trees.pack_parent.cpu().numpy()
        ids = np.random.default_rng(1000 + rank).choice(w.B, size=2, replace=False).tolist()
        for b in ids:
            q, k, v = (x.float() for x in _seq_inputs(w, st, b))
            words = [otree.ancestor_words(pp[cq[b]:cq[b + 1]])]
            S, P = w.S[b], w.P[b]
            outs[b] = oattn.tree_attention(q, k, v, [0, P], [0, S + P], [S], [P], words)
    errs = [(st.out[cq[b]:cq[b + 1]].float().cpu() - o).abs() for b, o in outs.items()]
    mx = max(e.max().item() for e in errs)
    mean = statistics.mean(e.mean().item() for e in errs)
    mx, = _max_over_ranks([mx], dev, world)
    n, = _max_over_ranks([float(len(outs))], dev, world, op="sum")
    return {"max_abs_err": mx, "mean_abs_err": round(mean, 7), "seqs_checked": int(n), "tolerance": TOL_BF16,
            "ok": bool(mx < TOL_BF16),
            "against": "fp32 CPU oracle of the masked-softmax reference on the same bf16 inputs and GPU trees"}


def config5_sweep(dev, world, rank, hbm, tf_burst, args):
    """Configuration 5 over the job's GPUs: one attention call per width, l(N), c1 and N*.

    One fixed batch of 512 sequences (prefix U[2048,16384], Qwen3-8B geometry, V=151936),
    sharded by sequence cost over the ranks (LPT, no collective on the path). Per width the
    trees are built on the GPU from block scores drawn on the device (normal, scale 5), then one
    ragged attention call over the rank's shard is timed (CUDA events, mean of `iters` after
    two warm-ups); l(N) is the max over ranks. c0/c1 are the least-squares line over
    16 <= n = N+1 <= 128 (the fit of cast_trees/width.py:22-27); predict_width of the reference
    package (baseline/_ref) turns the curve into the deployed width N*.
    """
    try:
        import cast_b200
        from cast_b200 import _lib, sharding, workloads
        base = workloads.config(5)
        costs = [sharding.sequence_cost(s, 129) for s in base.S]
        mine = sharding.lpt_shards(costs, world)[rank]
        sub = base.shard(mine)
        g = torch.Generator(device=dev).manual_seed(base.seed * 7919 + 17)
        logits = torch.empty((sub.B, 15, sub.V), dtype=torch.float64, device=dev)
        logits.normal_(generator=g).mul_(5.0)
        idx, lp = cast_b200.block_topk_device(logits, 8)
        del logits
        rows = []
        iters = args.config5_iters
        for N in WIDTHS:
            ww = workloads.with_width(sub, N)
            lay = ww.layout()
            t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
            cu_q = t(lay["cu_q"])
            trees = cast_b200.build_trees(idx, lp, N, 8, max_budget=N, cu_q=cu_q, total_q=lay["total_q"])
            q, k, v = ww.make_qkv(dev)
            out = torch.empty_like(q)
            a = (q, k, v, cu_q, t(lay["cu_kv"]), t(lay["prefix_len"]), t(lay["pack_len"]), None)
            kw = dict(parent=trees.pack_parent, max_pack=lay["max_pack"], max_kv=lay["max_kv"], out=out)
            for _ in range(2):
                cast_b200.varlen_tree_attention(*a, **kw)
            torch.cuda.synchronize()
            if world > 1:
                _dist().barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(iters):
                cast_b200.varlen_tree_attention(*a, **kw)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / iters
            depth_sums = trees.depth.sum(dim=1, dtype=torch.int64).cpu().tolist()
            fl, by = ww.attn_flops(depth_sums), ww.attn_bytes()
            ms, = _max_over_ranks([ms], dev, world)
            fl, by = _max_over_ranks([fl, by], dev, world, op="sum")
            t_h, t_t = by / (world * hbm * 1e9), fl / (world * tf_burst * 1e12)
            rows.append(dict(N=N, n=N + 1, ms=round(ms, 4), tflops=round(fl / (ms * 1e-3) / 1e12, 1),
                             gbs=round(by / (ms * 1e-3) / 1e9, 1), bound="tensor" if t_t >= t_h else "hbm",
                             frac=round(max(t_h, t_t) / (ms * 1e-3), 4)))
            del q, k, v, out, trees, a, kw
            torch.cuda.empty_cache()
        if _lib.device_error() != 0:
            return {"error": "device error in the configuration-5 sweep"}
        n = np.array([r["n"] for r in rows], float)
        ms = np.array([r["ms"] for r in rows], float)
        sel = (n >= 16) & (n <= 128)
        c1, c0 = np.polyfit(n[sel], ms[sel], 1)
        res = {"workload": f"config5: fixed B=512, prefix U[2048,16384], 32/8 heads, d=128, V=151936, "
                           f"LPT-sharded over {world} GPU(s) (strong scaling); one attention call per width",
               "batch": base.B, "shard_imbalance": round(sharding.imbalance(base.S, [129] * base.B,
                                                                           sharding.lpt_shards(costs, world)), 4),
               "iters": iters, "widths": [r["N"] for r in rows], "n": n.tolist(),
               "l_ms": [r["ms"] for r in rows], "tflops": [r["tflops"] for r in rows],
               "gbs": [r["gbs"] for r in rows], "bound": [r["bound"] for r in rows],
               "frac": [r["frac"] for r in rows], "frac_basis": "binding floor (HBM or burst bf16) / l(N)",
               "c0_ms": round(float(c0), 5), "c1_ms_per_packed_token": round(float(c1), 6)}
        res["predict_width"] = _predict_width(n.tolist(), ms.tolist())
        return res
    except Exception as e:
        return {"error": f"{type(e).__name__}: {e}"}


def _predict_width(n, ms):
    """cast_trees.width.predict_width of the installed reference package (default mass curve, no drafter time)."""
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "cast_trees" / "width.py").exists():
        return {"unavailable": "reference package not installed beside the repo (baseline/_ref)"}
    sys.path.insert(0, str(ref))
    try:
        from cast_trees.width import predict_width
        p = predict_width(n, ms)
        return {"c0_ms": round(p.c0, 5), "c1_ms_per_packed_token": round(p.c1, 6), "n_stop": int(p.n_stop),
                "n_star": int(p.n_star), "crossed": bool(p.crossed), "text": str(p)}
    except Exception as e:
        return {"unavailable": f"{type(e).__name__}: {e}"}
    finally:
        sys.path.remove(str(ref))


def run_reference(args):
    """The reference's CPU path (oracle port) on the host cores, one sampled sequence per step.

    Each step is a full verify round for one sequence of the same batch the cast arm runs
    (sequence step mod 64 of rank 0's shard): numpy tree build once, then `layers` attention
    calls. ms_per_step is the measured wall time of those steps; value = the attention flops
    they did / that time.
    """
    rank, world, local = _env()
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    w = rank_workload(0, world)
    g = torch.Generator().manual_seed(1234)
    times, flops = [], 0
    t_tree_all = t_attn_all = 0.0
    for i in range(args.warmup + args.steps):
        b = i % w.B
        S, P = w.S[b], w.P[b]
        qkv = ((torch.randn(P, w.H_q, w.D, generator=g) * 0.5).to(w.dtype),
               (torch.randn(S + P, w.H_kv, w.D, generator=g) * 0.5).to(w.dtype),
               (torch.randn(S + P, w.H_kv, w.D, generator=g) * 0.5).to(w.dtype))
        t0 = time.perf_counter()
        tt, ta, fl, _, _ = _cpu_round(w, b, args.layers, qkv)
        t1 = time.perf_counter()
        if i >= args.warmup:
            times.append(t1 - t0)
            flops += fl
            t_tree_all += tt
            t_attn_all += ta
    tot = sum(times)
    value = flops / tot / 1e12
    sample = (f"one sequence per step (sequence step mod {w.B} of the batch), a full round each: numpy "
              f"block_topk + heap build_tree (1 thread, {t_tree_all:.2f} s over the timed steps) and "
              f"{args.layers} fp32 masked-softmax attention calls (torch, all threads, {t_attn_all:.2f} s); "
              f"ms_per_step is the measured wall time of one such step")
    emit({
        "metric": METRIC, "impl": "reference", "value": round(value, 6), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * tot / max(1, args.steps), 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded normal(scale=5) block scores 15x128256 fp64, q/k/v N(0,1)*0.5 bf16",
        "config": bench_config(args, world),
        "cpu_baseline": {"value": round(value, 6), "unit": "TFLOP/s", "cores": torch.get_num_threads(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference's path is Python on the host (numpy tree builder, torch fp32 masked softmax); its "
                "only GPU piece, a Triton kernel, takes packs of at most 64 tokens and cannot run P=128",
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
    ap.add_argument("--layers", type=int, default=LAYERS_DEFAULT, help="attention calls per verify round")
    ap.add_argument("--cpu-seqs", type=int, default=2, help="sequences in the cpu_baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-config5", action="store_true")
    ap.add_argument("--config5-iters", type=int, default=5)
    ap.add_argument("--traffic-csv", default=None,
                    help="ncu --csv capture of attn_tc_kernel with dram__bytes_read/write.sum for roofline.traffic")
    args = ap.parse_args()
    if args.impl == "reference":
        args.warmup = max(args.warmup, 0)
        run_reference(args)
    else:
        args.warmup = max(args.warmup, 3)
        run_cast(args)


if __name__ == "__main__":
    main()
