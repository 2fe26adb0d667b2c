"""Seeded synthetic workloads of the benchmark configurations.

No datasets or checkpoints exist here, so every configuration is synthetic
with the stated shapes and distributions: for sequence b of configuration
seed s, ``np.random.default_rng([s, b, 0])`` draws the prefix length and then
the tree width, and ``np.random.default_rng([s, b, 1])`` the 15 x V drafter
block scores (normal, scale 5); q/k/v are i.i.d. normal times ``qkv_scale``
from a torch generator seeded from s.
Configuration 1 follows its own recipe exactly (rng(0) logits, a CPU torch
generator seeded 0 drawing q, k, v in that order).
"""
from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np
import torch

L_BLOCK = 15      # future positions scored by the block drafter
TOPK = 8          # branch factor k


@dataclass
class Workload:
    name: str
    seed: int
    V: int
    S: List[int]                  # prefix length per sequence
    N: List[int]                  # non-root tree nodes per sequence
    dtype: torch.dtype = torch.bfloat16
    H_q: int = 32
    H_kv: int = 8
    D: int = 128
    qkv_scale: float = 0.5
    cfg1_recipe: bool = False
    seq_ids: Optional[List[int]] = None   # global sequence ids (a shard keeps the parent's ids)
    _layout: dict = field(default_factory=dict, repr=False)

    @property
    def B(self):
        return len(self.S)

    @property
    def P(self):
        return [n + 1 for n in self.N]

    def ids(self):
        return self.seq_ids if self.seq_ids is not None else list(range(self.B))

    def logits(self, b):
        """fp64 [15, V] block scores of local sequence b (numpy)."""
        if self.cfg1_recipe:
            return np.random.default_rng(0).normal(scale=5, size=(L_BLOCK, self.V))
        rng = np.random.default_rng([self.seed, self.ids()[b], 1])
        return rng.normal(scale=5, size=(L_BLOCK, self.V))

    def logits_batch(self, out=None):
        """fp64 [B, 15, V] (numpy, or filled into a given host tensor)."""
        arr = out if out is not None else np.empty((self.B, L_BLOCK, self.V), dtype=np.float64)
        for b in range(self.B):
            arr[b] = self.logits(b) if not isinstance(arr, torch.Tensor) else torch.from_numpy(self.logits(b))
        return arr

    def layout(self):
        if not self._layout:
            P = np.array(self.P, dtype=np.int64)
            S = np.array(self.S, dtype=np.int64)
            cu_q = np.concatenate([[0], np.cumsum(P)]).astype(np.int32)
            cu_kv = np.concatenate([[0], np.cumsum(S + P)]).astype(np.int32)
            self._layout = dict(cu_q=cu_q, cu_kv=cu_kv, prefix_len=S.astype(np.int32),
                                pack_len=P.astype(np.int32), total_q=int(cu_q[-1]),
                                total_kv=int(cu_kv[-1]), max_pack=int(P.max()), max_kv=int((S + P).max()))
        return self._layout

    def make_qkv(self, device, dtype=None):
        dtype = dtype or self.dtype
        lay = self.layout()
        if self.cfg1_recipe:
            g = torch.Generator().manual_seed(0)
            q = torch.randn(lay["total_q"], self.H_q, self.D, generator=g)
            k = torch.randn(lay["total_kv"], self.H_kv, self.D, generator=g)
            v = torch.randn(lay["total_kv"], self.H_kv, self.D, generator=g)
            return q.to(device, dtype), k.to(device, dtype), v.to(device, dtype)
        g = torch.Generator(device=device).manual_seed(self.seed * 1000003 + (self.ids()[0] if self.B else 0))
        out = []
        for rows, heads in ((lay["total_q"], self.H_q), (lay["total_kv"], self.H_kv), (lay["total_kv"], self.H_kv)):
            t = torch.empty(rows, heads, self.D, dtype=torch.float32, device=device)
            t.normal_(generator=g).mul_(self.qkv_scale)
            out.append(t.to(dtype))
        return tuple(out)

    # algorithmic work (the roofline basis)
    def attn_bytes(self):
        e = torch.tensor([], dtype=self.dtype).element_size()
        return sum((s + p) * self.H_kv * self.D * 2 * e + 2 * p * self.H_q * self.D * e
                   for s, p in zip(self.S, self.P))

    def attn_flops(self, depth_sums):
        """4 * H_q * D * (P*S + sum |anc|); |anc| of pack token i = depth_i + 1."""
        tot = 0
        for s, p, ds in zip(self.S, self.P, depth_sums):
            tot += 4 * self.H_q * self.D * (p * s + p + int(ds))
        return tot

    def topk_bytes(self):
        return self.B * L_BLOCK * self.V * 8

    def shard(self, ranks):
        """Local sub-workload of the given global sequence indices."""
        ids = self.ids()
        return Workload(self.name, self.seed, self.V, [self.S[i] for i in ranks], [self.N[i] for i in ranks],
                        self.dtype, self.H_q, self.H_kv, self.D, self.qkv_scale, self.cfg1_recipe,
                        [ids[i] for i in ranks])


def _ragged(seed, B, s_lo, s_hi, widths):
    S, N = [], []
    for b in range(B):
        rng = np.random.default_rng([seed, b, 0])
        S.append(int(rng.integers(s_lo, s_hi + 1)))
        N.append(int(widths[int(rng.integers(0, len(widths)))]))
    return S, N


def config(n, dtype=None):
    """Benchmark configuration n (1..5) of the recipe in this module's docstring."""
    if n == 1:
        return Workload("config1", 0, 64, [512], [16], dtype or torch.float32, qkv_scale=1.0, cfg1_recipe=True)
    if n == 2:
        S, N = _ragged(1, 16, 256, 4096, (16, 24, 32, 48, 64, 96, 128))
        return Workload("config2", 1, 151936, S, N, dtype or torch.bfloat16)
    if n == 3:
        S, N = _ragged(2, 64, 4096, 8192, (127,))
        return Workload("config3", 2, 128256, S, N, dtype or torch.bfloat16)
    if n == 4:
        return Workload("config4", 3, 151936, [32768] * 8, [128] * 8, dtype or torch.bfloat16)
    if n == 5:
        S, N = _ragged(4, 512, 2048, 16384, (16, 24, 32, 48, 64, 96, 128, 256))
        return Workload("config5", 4, 151936, S, N, dtype or torch.bfloat16)
    raise ValueError(n)


def with_width(w, n_nodes):
    """The same sequences at a fixed tree width (the l(N) sweep of configuration 5)."""
    return Workload(w.name + f"_N{n_nodes}", w.seed, w.V, list(w.S), [n_nodes] * w.B, w.dtype, w.H_q, w.H_kv,
                    w.D, w.qkv_scale, w.cfg1_recipe, w.seq_ids)
