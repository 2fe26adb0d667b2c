"""The allocation-free attention entry point, called through the C ABI.

cast_tree_attn_fwd_noalloc serves callers that may not allocate device memory
(a host that owns every allocation, a strict memory budget): when the key range
is split, its partial results live in a fixed scratch array inside the library
instead of a caller-provided workspace. This file is collected last on purpose,
so a run that stops at the first failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

import cast_b200
from cast_b200 import _lib

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2   # the bf16 bound the other attention tests use


def _problem(dev):
    """Two sequences with long prefixes: the launch splits keys and needs scratch."""
    g = torch.Generator().manual_seed(77)
    rng = np.random.default_rng(77)
    S, P = [16384, 8000], [65, 17]
    Hq, Hkv, D = 32, 8, 128
    parents = []
    for p in P:
        parents += [-1] + [int(rng.integers(0, i)) for i in range(1, p)]
    tq, tkv = sum(P), sum(s + p for s, p in zip(S, P))
    q = (torch.randn(tq, Hq, D, generator=g) * 0.5).to(dev, torch.bfloat16)
    k = (torch.randn(tkv, Hkv, D, generator=g) * 0.5).to(dev, torch.bfloat16)
    v = (torch.randn(tkv, Hkv, D, generator=g) * 0.5).to(dev, torch.bfloat16)
    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device=dev)
    return dict(q=q, k=k, v=v, cu_q=i32([0, P[0], P[0] + P[1]]), cu_kv=i32([0, S[0] + P[0], tkv]),
                prefix=i32(S), pack=i32(P), parent=i32(parents), B=2, total_q=tq, total_kv=tkv,
                Hq=Hq, Hkv=Hkv, D=D, max_pack=max(P), max_kv=max(s + p for s, p in zip(S, P)))


def _noalloc(L, pr, out):
    strides = (ctypes.c_int64 * 12)(*pr["q"].stride(), *pr["k"].stride(), *pr["v"].stride(), *out.stride())
    return L.cast_tree_attn_fwd_noalloc(
        pr["q"].data_ptr(), pr["k"].data_ptr(), pr["v"].data_ptr(), out.data_ptr(), _lib.CAST_BF16,
        ctypes.addressof(strides), pr["cu_q"].data_ptr(), pr["cu_kv"].data_ptr(), pr["prefix"].data_ptr(),
        pr["pack"].data_ptr(), None, 0, pr["parent"].data_ptr(), pr["B"], pr["total_q"], pr["total_kv"],
        pr["Hq"], pr["Hkv"], pr["D"], 0.0, pr["max_pack"], pr["max_kv"],
        torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_the_workspace_entry_point_twice(cuda):
    L = _lib.lib()
    pr = _problem(cuda)
    need = cast_b200.workspace_size(torch.bfloat16, pr["B"], pr["total_q"], pr["Hq"], pr["Hkv"], pr["D"],
                                    pr["max_pack"], pr["max_kv"])
    assert 0 < need <= _lib.CAST_NOALLOC_SCRATCH_BYTES      # this problem really uses the scratch
    ref = cast_b200.varlen_tree_attention(pr["q"], pr["k"], pr["v"], pr["cu_q"], pr["cu_kv"], pr["prefix"],
                                          pr["pack"], None, parent=pr["parent"], max_pack=pr["max_pack"],
                                          max_kv=pr["max_kv"])
    assert _lib.device_error() == 0
    for _ in range(2):                                      # the second call reuses the same scratch
        out = torch.full_like(pr["q"], float("nan"))
        assert _noalloc(L, pr, out) == 0
        assert _lib.device_error() == 0
        err = (out.float() - ref.float()).abs().max().item()
        assert err < BF16_TOL, err


def test_noalloc_rejects_problems_beyond_its_scratch(cuda):
    # 18 sequences of 8192-token prefixes and 128-token packs: 288 (sequence, KV head, row block)
    # units, fewer than two per SM, so the launch splits the keys in two, and the fp32 partials
    # (2 x 2304 rows x 32 heads x 130 floats, 76.7 MB) exceed the fixed array: rejected before any launch
    L = _lib.lib()
    B, S, P, Hq, Hkv, D = 18, 8192, 128, 32, 8, 128
    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device=cuda)
    q = torch.empty(B * P, Hq, D, dtype=torch.bfloat16, device=cuda)
    k = torch.empty(B * (S + P), Hkv, D, dtype=torch.bfloat16, device=cuda)
    v = torch.empty_like(k)
    pr = dict(q=q, k=k, v=v, cu_q=i32([b * P for b in range(B + 1)]),
              cu_kv=i32([b * (S + P) for b in range(B + 1)]), prefix=i32([S] * B), pack=i32([P] * B),
              parent=i32(([-1] + list(range(P - 1))) * B), B=B, total_q=B * P, total_kv=B * (S + P),
              Hq=Hq, Hkv=Hkv, D=D, max_pack=P, max_kv=S + P)
    need = cast_b200.workspace_size(torch.bfloat16, B, B * P, Hq, Hkv, D, P, S + P)
    assert need > _lib.CAST_NOALLOC_SCRATCH_BYTES
    out = torch.zeros_like(q)
    assert _noalloc(L, pr, out) == -12                    # CAST_ERR_SCRATCH_LIMIT
    assert b"scratch" in L.cast_strerror(-12)
    assert _lib.device_error() == 0
    assert torch.count_nonzero(out).item() == 0            # nothing was launched
