"""Tree attention reading the prefix in place from per-request KV stores.

The store layout is the serving loop's (cast_trees/serving.py:190-205):
[B, H_kv, S_max, D] per layer, request b's prefix in rows [0, S_b); the pack
K/V are the pass's own [total_q, H_kv, D] rows (here, like the hook's
key[0].transpose(0, 1), a strided view). Checked against the fp32 oracle on the
assembled ragged layout and against the regular entry point.
"""
import numpy as np
import pytest
import torch

import cast_b200
from cast_b200 import _lib
from oracle import attn as oattn
from oracle import tree as otree

pytestmark = pytest.mark.gpu


def _store_case(seed, S_list, P_list, Hq=32, Hkv=8, D=128, dtype=torch.bfloat16, dev="cuda", poison=True):
    g = torch.Generator().manual_seed(seed)
    rng = np.random.default_rng(seed)
    B = len(S_list)
    S_max = max(S_list) + 37
    k_store = torch.randn(B, Hkv, S_max, D, generator=g) * 0.5
    v_store = torch.randn(B, Hkv, S_max, D, generator=g) * 0.5
    if poison:      # rows past each prefix hold non-finite garbage: never read into the result
        for b, s in enumerate(S_list):
            k_store[b, :, s:] = float("nan")
            v_store[b, :, s:] = float("inf")
    total_q = sum(P_list)
    q = torch.randn(total_q, Hq, D, generator=g) * 0.5
    kp_hm = torch.randn(Hkv, total_q, D, generator=g) * 0.5    # the hook's [H_kv, T, D] layout
    vp_hm = torch.randn(Hkv, total_q, D, generator=g) * 0.5
    parents = []
    for p in P_list:
        parents += [-1] + [int(rng.integers(max(0, i - 9), i)) for i in range(1, p)]
    cu_q = np.concatenate([[0], np.cumsum(P_list)]).astype(np.int32)
    return dict(q=q, k_store=k_store, v_store=v_store, kp_hm=kp_hm, vp_hm=vp_hm, cu_q=cu_q,
                S=np.array(S_list, np.int32), P=np.array(P_list, np.int32), parent=np.array(parents, np.int32))


def _oracle(c, dtype):
    S, P, cu_q = c["S"], c["P"], c["cu_q"]
    ks, vs, qs = [], [], []
    kp = c["kp_hm"].transpose(0, 1)
    vp = c["vp_hm"].transpose(0, 1)
    for b in range(len(S)):
        ks += [c["k_store"][b, :, :S[b]].transpose(0, 1), kp[cu_q[b]:cu_q[b] + P[b]]]
        vs += [c["v_store"][b, :, :S[b]].transpose(0, 1), vp[cu_q[b]:cu_q[b] + P[b]]]
    k = torch.cat(ks).to(dtype).float()
    v = torch.cat(vs).to(dtype).float()
    cu_kv = np.concatenate([[0], np.cumsum(S + P)])
    words = [otree.ancestor_words(c["parent"][cu_q[b]:cu_q[b + 1]]) for b in range(len(S))]
    return oattn.tree_attention(c["q"].to(dtype).float(), k, v, cu_q, cu_kv, S, P, words), k, v, cu_kv


def _run_store(c, dev, dtype, **kw):
    t = lambda a: torch.from_numpy(np.asarray(a)).to(dev)
    kp = c["kp_hm"].to(dev, dtype).transpose(0, 1)     # strided view, as the hook would pass it
    vp = c["vp_hm"].to(dev, dtype).transpose(0, 1)
    out = cast_b200.varlen_tree_attention_store(c["q"].to(dev, dtype), c["k_store"].to(dev, dtype),
                                                c["v_store"].to(dev, dtype), kp, vp, t(c["cu_q"]), t(c["S"]),
                                                t(c["P"]), None, parent=t(c["parent"]), **kw)
    assert _lib.device_error() == 0
    return out


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_store_matches_oracle(cuda, dtype):
    # S = 0, S a multiple of 128, S ending inside a tile; P = 1, 128, 129, 300
    c = _store_case(31, [0, 128, 257, 1000, 4099], [64, 1, 129, 300, 128])
    got = _run_store(c, cuda, dtype).float().cpu()
    ref, *_ = _oracle(c, dtype)
    assert torch.isfinite(got).all()
    err = (got - ref).abs().max().item()
    assert err < 2e-2, err


def test_store_matches_regular_entry_point(cuda):
    c = _store_case(32, [300, 0, 777, 129], [50, 20, 128, 65], poison=False)
    got = _run_store(c, cuda, torch.bfloat16)
    _, k, v, cu_kv = _oracle(c, torch.bfloat16)
    t = lambda a: torch.from_numpy(np.asarray(a, dtype=np.int32)).to(cuda)
    reg = cast_b200.varlen_tree_attention(c["q"].to(cuda, torch.bfloat16), k.to(cuda, torch.bfloat16),
                                          v.to(cuda, torch.bfloat16), t(c["cu_q"]), t(cu_kv), t(c["S"]), t(c["P"]),
                                          None, parent=t(c["parent"]))
    assert (got.float() - reg.float()).abs().max().item() < 2e-2


@pytest.mark.parametrize("Hq,Hkv", [(8, 8), (16, 8), (64, 4)])
def test_store_head_groups_and_split_keys(cuda, Hq, Hkv):
    # two sequences with long prefixes: the launch splits the key tiles
    c = _store_case(33, [20000, 9000], [129, 17], Hq=Hq, Hkv=Hkv)
    got = _run_store(c, cuda, torch.bfloat16).float().cpu()
    ref, *_ = _oracle(c, torch.bfloat16)
    assert (got - ref).abs().max().item() < 2e-2


@pytest.mark.parametrize("path", ["split", "exact"])
def test_store_fp32(cuda, path):
    # fp32 as the reference hook passes it: the split path reads the stores in its split pass (rows past
    # each prefix are non-finite and never read); the exact path assembles the ragged layout on the device
    c = _store_case(34, [100, 3, 0, 1280, 4099], [10, 7, 130, 64, 1], Hq=8, Hkv=2)
    got = _run_store(c, cuda, torch.float32, fp32_path=path).cpu()
    ref, *_ = _oracle(c, torch.float32)
    assert torch.isfinite(got).all()
    assert (got - ref).abs().max().item() < 1e-4


def test_store_fp32_split_with_key_splits(cuda):
    c = _store_case(36, [20000, 9000], [129, 17])
    got = _run_store(c, cuda, torch.float32).cpu()
    ref, *_ = _oracle(c, torch.float32)
    assert (got - ref).abs().max().item() < 1e-4


@pytest.mark.parametrize("D,Hq,Hkv", [(64, 8, 2), (128, 12, 4)])
def test_store_shapes_outside_the_tensor_core_kernel(cuda, D, Hq, Hkv):
    # head dim 64 / group size 3: assembled on the device (cast_kv_ragged_gather), then the CUDA-core kernel
    c = _store_case(37, [300, 0, 129], [20, 33, 5], Hq=Hq, Hkv=Hkv, D=D)
    got = _run_store(c, cuda, torch.bfloat16).float().cpu()
    ref, *_ = _oracle(c, torch.bfloat16)
    assert torch.isfinite(got).all()
    assert (got - ref).abs().max().item() < 2e-2


def test_store_with_unaligned_row_stride(cuda):
    # a store whose row stride (132 elements) is not a 16-byte multiple: no TMA map, the device assembly
    c = _store_case(38, [257, 40], [31, 129])
    wide = torch.zeros(2, 8, c["k_store"].shape[2], 132, dtype=torch.bfloat16, device=cuda)
    ks, vs = wide.clone(), wide.clone()
    ks[..., :128] = c["k_store"].to(cuda, torch.bfloat16)
    vs[..., :128] = c["v_store"].to(cuda, torch.bfloat16)
    t = lambda a: torch.from_numpy(np.asarray(a)).to(cuda)
    out = cast_b200.varlen_tree_attention_store(c["q"].to(cuda, torch.bfloat16), ks[..., :128], vs[..., :128],
                                                c["kp_hm"].to(cuda, torch.bfloat16).transpose(0, 1),
                                                c["vp_hm"].to(cuda, torch.bfloat16).transpose(0, 1), t(c["cu_q"]),
                                                t(c["S"]), t(c["P"]), None, parent=t(c["parent"]))
    assert _lib.device_error() == 0
    ref, *_ = _oracle(c, torch.bfloat16)
    assert (out.float().cpu() - ref).abs().max().item() < 2e-2


def test_ragged_gather_layout(cuda):
    import ctypes
    c = _store_case(39, [5, 0, 130], [3, 2, 4], Hq=8, Hkv=2, D=64)
    dev = cuda
    t = lambda a: torch.from_numpy(np.asarray(a)).to(dev)
    ks, vs = c["k_store"].to(dev), c["v_store"].to(dev)
    kp, vp = c["kp_hm"].to(dev).transpose(0, 1), c["vp_hm"].to(dev).transpose(0, 1)
    rows_cap = 3 * (130 + 4)
    k_rag = torch.full((rows_cap, 2, 64), 7.0, device=dev)
    v_rag = torch.full_like(k_rag, 7.0)
    cu_kv = torch.empty(4, dtype=torch.int32, device=dev)
    st = (ctypes.c_int64 * 14)(*ks.stride(), *vs.stride(), *kp.stride(), *vp.stride())
    cu_q, S, P = t(c["cu_q"]), t(c["S"]), t(c["P"])    # held: the call takes raw device pointers
    rc = _lib.lib().cast_kv_ragged_gather(ks.data_ptr(), vs.data_ptr(), kp.data_ptr(), vp.data_ptr(), 4,
                                          ctypes.addressof(st), cu_q.data_ptr(), S.data_ptr(),
                                          P.data_ptr(), 3, 9, 3, ks.shape[2], 2, 64, 4, rows_cap,
                                          k_rag.data_ptr(), v_rag.data_ptr(), cu_kv.data_ptr(),
                                          torch.cuda.current_stream().cuda_stream)
    assert rc == 0 and _lib.device_error() == 0
    _, k_ref, v_ref, cu_ref = _oracle(c, torch.float32)
    n = int(cu_ref[-1])
    assert cu_kv.cpu().tolist() == [int(x) for x in cu_ref]
    assert torch.equal(k_rag[:n].cpu(), k_ref) and torch.equal(v_rag[:n].cpu(), v_ref)
    assert torch.all(k_rag[n:] == 0) and torch.all(v_rag[n:] == 0)


def test_store_with_ancestor_bits_as_the_hook_passes_them(cuda):
    # the serving hook passes 64-bit ancestor words (cast_trees/serving.py:213-222), q as a strided view
    c = _store_case(35, [300, 70, 1000], [40, 64, 9], poison=False)
    bits = np.concatenate([otree.ancestor_words(c["parent"][int(a):int(b)]).reshape(-1)
                           for a, b in zip(c["cu_q"][:-1], c["cu_q"][1:])]).astype(np.uint64).view(np.int64)
    t = lambda a: torch.from_numpy(np.asarray(a)).to(cuda)
    q_hm = c["q"].to(cuda, torch.bfloat16).transpose(0, 1).contiguous().transpose(0, 1)   # [T, H_q, D] view
    out = cast_b200.varlen_tree_attention_store(q_hm, c["k_store"].to(cuda, torch.bfloat16),
                                                c["v_store"].to(cuda, torch.bfloat16),
                                                c["kp_hm"].to(cuda, torch.bfloat16).transpose(0, 1),
                                                c["vp_hm"].to(cuda, torch.bfloat16).transpose(0, 1), t(c["cu_q"]),
                                                t(c["S"]), t(c["P"]), t(bits))
    assert _lib.device_error() == 0
    ref, *_ = _oracle(c, torch.bfloat16)
    assert (out.float().cpu() - ref).abs().max().item() < 2e-2
