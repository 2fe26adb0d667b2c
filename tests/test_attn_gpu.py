"""Tree attention on the GPU (through the C ABI) against the CPU oracle.

Tolerances (max abs error against the fp32 oracle on the same inputs):
fp32 inputs 1e-4, bf16 / fp16 inputs 2e-2, the path's stated bounds; the
reference test's own bound (max 5e-2, mean 5e-3) is also checked for the
reference scenario.
"""
import numpy as np
import pytest
import torch

import cast_b200
from cast_b200 import _lib, workloads
from oracle import attn as oattn
from oracle import tree as otree
from tests.golden.make_golden import ragged_scenario

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2, torch.float16: 2e-2}


def _words(sc):
    """Per-sequence ancestor words from the scenario's pack parents."""
    cu = sc["cu_q"].tolist()
    return [otree.ancestor_words(sc["parent"][cu[b]:cu[b + 1]]) for b in range(len(cu) - 1)]


def _run(sc, dtype, dev, mode="parent", **kw):
    q, k, v = (sc[n].to(dev, dtype) for n in ("q", "k", "v"))
    args = (q, k, v, sc["cu_q"].to(dev), sc["cu_kv"].to(dev), torch.as_tensor(sc["prefix"]).to(dev),
            torch.as_tensor(sc["pack"]).to(dev))
    if mode == "parent":
        out = cast_b200.varlen_tree_attention(*args, None, parent=torch.as_tensor(sc["parent"]).to(dev), **kw)
    else:
        out = cast_b200.varlen_tree_attention(*args, torch.as_tensor(sc["bits"]).to(dev), **kw)
    assert _lib.device_error() == 0
    return out


def _oracle(sc, dtype):
    q, k, v = (sc[n].to(dtype).float() for n in ("q", "k", "v"))
    return oattn.tree_attention(q, k, v, sc["cu_q"], sc["cu_kv"], sc["prefix"], sc["pack"], _words(sc))


# fp32 inputs run two kernels: the tensor-core path from the three-term bf16 split (the default)
# and the exact CUDA-core kernel; both are held to 1e-4
DTYPE_PATHS = [(torch.float32, "split"), (torch.float32, "exact"), (torch.bfloat16, "split")]


@pytest.mark.parametrize("dtype,path", DTYPE_PATHS)
@pytest.mark.parametrize("mode", ["bits", "parent"])
def test_reference_scenario(cuda, dtype, path, mode):
    # tests/test_tree_attn.py:11-37 scenario: B=8, 32/8 heads, D=128, S in [200,400), P in [2,64)
    sc = ragged_scenario(seed=0, B=8, Hq=32, Hkv=8, D=128, s_range=(200, 400), p_range=(2, 64))
    got = _run(sc, dtype, cuda, mode, fp32_path=path).float().cpu()
    err = (got - _oracle(sc, dtype)).abs()
    assert err.max().item() < TOL[dtype], err.max().item()
    assert err.mean().item() < 5e-3


@pytest.mark.parametrize("path", ["split", "exact"])
def test_golden_config1_fp32(cuda, golden, path):
    g = golden("attn_cfg1.npz")
    w = workloads.config(1)
    q, k, v = w.make_qkv(cuda)
    lay = w.layout()
    parent = torch.from_numpy(otree.pack_parent(g["parent"])).to(cuda)
    out = cast_b200.varlen_tree_attention(q, k, v, torch.from_numpy(lay["cu_q"]).to(cuda),
                                          torch.from_numpy(lay["cu_kv"]).to(cuda),
                                          torch.from_numpy(lay["prefix_len"]).to(cuda),
                                          torch.from_numpy(lay["pack_len"]).to(cuda), None, parent=parent,
                                          fp32_path=path)
    err = (out.cpu() - torch.from_numpy(g["out"])).abs().max().item()
    assert err < 1e-4, err


@pytest.mark.parametrize("path", ["split", "exact"])
@pytest.mark.parametrize("mode", ["bits", "parent"])
def test_golden_ragged_fp32(cuda, golden, mode, path):
    g = golden("attn_ragged.npz")
    sc = ragged_scenario(int(g["seed"]))
    got = _run(sc, torch.float32, cuda, mode, fp32_path=path).cpu()
    err = (got - torch.from_numpy(g["out"])).abs().max().item()
    assert err < 1e-4, err


def test_bits_and_parent_agree_exactly(cuda):
    sc = ragged_scenario(seed=3, B=5, Hq=16, Hkv=4, D=128)
    a = _run(sc, torch.bfloat16, cuda, "bits")
    b = _run(sc, torch.bfloat16, cuda, "parent")
    assert torch.equal(a, b)


def _tree_scenario(seed, B, S_list, P_list, Hq=32, Hkv=8, D=128, depth_cap=None):
    g = torch.Generator().manual_seed(seed)
    rng = np.random.default_rng(seed)
    qs, ks, vs, parents = [], [], [], []
    cu_q, cu_kv = [0], [0]
    for S, P in zip(S_list, P_list):
        par = [-1]
        for i in range(1, P):
            lo = 0 if depth_cap is None else max(0, i - depth_cap)
            par.append(int(rng.integers(lo, i)))
        parents += par
        qs.append(torch.randn(P, Hq, D, generator=g))
        ks.append(torch.randn(S + P, Hkv, D, generator=g))
        vs.append(torch.randn(S + P, Hkv, D, generator=g))
        cu_q.append(cu_q[-1] + P)
        cu_kv.append(cu_kv[-1] + S + P)
    return dict(q=torch.cat(qs), k=torch.cat(ks), v=torch.cat(vs),
                cu_q=torch.tensor(cu_q, dtype=torch.int32), cu_kv=torch.tensor(cu_kv, dtype=torch.int32),
                prefix=np.array(S_list, np.int32), pack=np.array(P_list, np.int32),
                parent=np.array(parents, np.int32))


@pytest.mark.parametrize("dtype,path", DTYPE_PATHS)
def test_wide_packs_multiword(cuda, dtype, path):
    # P above 64 needs several ancestor words per token; the reference caps P at 64
    sc = _tree_scenario(5, 4, [300, 0, 1000, 77], [128, 257, 129, 1000])
    got = _run(sc, dtype, cuda, "parent", fp32_path=path).float().cpu()
    err = (got - _oracle(sc, dtype)).abs().max().item()
    assert err < TOL[dtype], err


@pytest.mark.parametrize("dtype,path", DTYPE_PATHS)
def test_long_prefix_split_kv(cuda, dtype, path):
    # few (sequence, head) pairs and a long prefix: the launch splits the keys
    sc = _tree_scenario(6, 2, [32768, 20000], [129, 17], Hq=32, Hkv=8)
    sc["q"] *= 0.5; sc["k"] *= 0.5; sc["v"] *= 0.5
    B, total_q = 2, int(sc["cu_q"][-1])
    assert cast_b200.workspace_size(dtype, B, total_q, 32, 8, 128, 129, 32768 + 129, fp32_path=path) > 0
    got = _run(sc, dtype, cuda, "parent", fp32_path=path).float().cpu()
    err = (got - _oracle(sc, dtype)).abs().max().item()
    assert err < TOL[dtype], err


@pytest.mark.parametrize("D,Hq,Hkv", [(64, 8, 8), (128, 8, 1), (64, 12, 4)])
def test_head_dims_and_groups(cuda, D, Hq, Hkv):
    sc = _tree_scenario(7, 3, [50, 513, 0], [3, 64, 40], Hq=Hq, Hkv=Hkv, D=D)
    for dtype in (torch.float32, torch.float16):
        got = _run(sc, dtype, cuda, "parent").float().cpu()
        err = (got - _oracle(sc, dtype)).abs().max().item()
        assert err < TOL[dtype], (dtype, err)


def test_strided_inputs(cuda):
    # k / v as head slices of a fused [T, 2*H_kv, D] buffer, q head-major transposed
    sc = _tree_scenario(8, 3, [100, 200, 10], [20, 5, 33], Hq=16, Hkv=4, D=128)
    kv = torch.cat([sc["k"], sc["v"]], dim=1).to(cuda)
    k, v = kv[:, :4], kv[:, 4:]
    q = sc["q"].transpose(0, 1).contiguous().to(cuda).transpose(0, 1)
    assert not k.is_contiguous() and not q.is_contiguous()
    out = cast_b200.varlen_tree_attention(q, k, v, sc["cu_q"].to(cuda), sc["cu_kv"].to(cuda),
                                          torch.as_tensor(sc["prefix"]).to(cuda),
                                          torch.as_tensor(sc["pack"]).to(cuda), None,
                                          parent=torch.as_tensor(sc["parent"]).to(cuda))
    err = (out.cpu() - _oracle(sc, torch.float32)).abs().max().item()
    assert err < 1e-4, err


def test_rows_that_see_nothing_are_zero(cuda):
    # S = 0 and a row whose ancestor word is empty: the reference writes 0 (tree_attn.py:89)
    q = torch.randn(3, 8, 128, device=cuda)
    k = torch.randn(3, 2, 128, device=cuda)
    v = torch.randn(3, 2, 128, device=cuda)
    bits = torch.tensor([0, 3, 7], dtype=torch.int64, device=cuda)
    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device=cuda)
    out = cast_b200.varlen_tree_attention(q, k, v, i32([0, 3]), i32([0, 3]), i32([0]), i32([3]), bits)
    assert torch.all(out[0] == 0)
    ref = oattn.tree_attention(q.cpu(), k.cpu(), v.cpu(), [0, 3], [0, 3], [0], [3], bits.cpu().numpy())
    assert (out.cpu() - ref).abs().max().item() < 1e-4


def test_sm_scale_and_empty_batch(cuda):
    sc = _tree_scenario(9, 2, [64, 65], [9, 10], Hq=8, Hkv=2, D=64)
    got = _run(sc, torch.float32, cuda, "parent", sm_scale=0.3).cpu()
    q, k, v = sc["q"], sc["k"], sc["v"]
    ref = oattn.tree_attention(q, k, v, sc["cu_q"], sc["cu_kv"], sc["prefix"], sc["pack"], _words(sc), sm_scale=0.3)
    assert (got - ref).abs().max().item() < 1e-4
    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device=cuda)
    z = torch.zeros(0, 8, 64, device=cuda)
    out = cast_b200.varlen_tree_attention(z, torch.zeros(0, 2, 64, device=cuda), torch.zeros(0, 2, 64, device=cuda),
                                          i32([0]), i32([0]), i32([]), i32([]), None,
                                          parent=i32([]), max_pack=0, max_kv=0)
    assert out.shape == (0, 8, 64)


def test_bad_parent_is_reported_not_fatal(cuda):
    # a parent array that is not in pack order: the kernel records the fault and the context stays usable
    sc = _tree_scenario(10, 1, [16], [8], Hq=8, Hkv=2, D=64)
    sc["parent"][5] = 6
    q, k, v = (sc[n].to(cuda) for n in ("q", "k", "v"))
    cast_b200.varlen_tree_attention(q, k, v, sc["cu_q"].to(cuda), sc["cu_kv"].to(cuda),
                                    torch.as_tensor(sc["prefix"]).to(cuda), torch.as_tensor(sc["pack"]).to(cuda),
                                    None, parent=torch.as_tensor(sc["parent"]).to(cuda))
    assert _lib.device_error() == 2          # CAST_DEV_BAD_PARENT
    assert _lib.device_error() == 0          # read-and-clear


def test_lengths_above_bounds_are_reported(cuda):
    # pack_len above the max_pack the caller promised: skipped and reported, no out-of-range access
    sc = _tree_scenario(11, 2, [16, 16], [8, 8], Hq=8, Hkv=2, D=64)
    q, k, v = (sc[n].to(cuda) for n in ("q", "k", "v"))
    cast_b200.varlen_tree_attention(q, k, v, sc["cu_q"].to(cuda), sc["cu_kv"].to(cuda),
                                    torch.as_tensor(sc["prefix"]).to(cuda), torch.as_tensor(sc["pack"]).to(cuda),
                                    None, parent=torch.as_tensor(sc["parent"]).to(cuda), max_pack=4, max_kv=24)
    assert _lib.device_error() == 1          # CAST_DEV_BAD_LAYOUT


def test_host_argument_errors(cuda):
    q = torch.randn(4, 6, 64, device=cuda)
    k = torch.randn(4, 4, 64, device=cuda)
    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device=cuda)
    with pytest.raises(AssertionError):
        cast_b200.varlen_tree_attention(q, k, k, i32([0, 4]), i32([0, 4]), i32([0]), i32([4]),
                                        torch.zeros(4, dtype=torch.int64, device=cuda))
    with pytest.raises(ValueError):
        cast_b200.varlen_tree_attention(q, k[:, :2], k[:, :2], i32([0, 4]), i32([0, 4]), i32([0]), i32([4]), None)


@pytest.mark.parametrize("Hq,Hkv", [(32, 8), (8, 8), (16, 8), (32, 4), (64, 4)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_tensor_core_kernel_shapes(cuda, Hq, Hkv, dtype):
    # ragged edge cases on the tcgen05 path: a pure pack (S = 0), a one-token
    # pack, a prefix that ends inside a key tile, row blocks with one query
    # tile, and packs wider than 64 tokens
    S_list = [0, 1, 127, 129, 700, 64, 2000]
    P_list = [70, 1, 33, 128, 300, 129, 17]
    sc = _tree_scenario(21, len(S_list), S_list, P_list, Hq=Hq, Hkv=Hkv, D=128)
    q, k, v = (sc[n].to(cuda, dtype) for n in ("q", "k", "v"))
    kind, _, _ = cast_b200.attention_plan(q, k, v, torch.empty_like(q), len(S_list), max(P_list),
                                          max(s + p for s, p in zip(S_list, P_list)))
    assert kind == "tcgen05"
    got = _run(sc, dtype, cuda, "parent").float().cpu()
    err = (got - _oracle(sc, dtype)).abs().max().item()
    assert err < TOL[dtype], err


def test_tensor_core_and_cuda_core_agree(cuda):
    # the same bf16 problem through both kernels (a non-multiple-of-8 head
    # stride sends the second call to the CUDA-core kernel)
    sc = _tree_scenario(22, 4, [1000, 37, 4096, 5], [128, 64, 100, 1], Hq=32, Hkv=8)
    q, k, v = (sc[n].to(cuda, torch.bfloat16) for n in ("q", "k", "v"))
    args = (sc["cu_q"].to(cuda), sc["cu_kv"].to(cuda), torch.as_tensor(sc["prefix"]).to(cuda),
            torch.as_tensor(sc["pack"]).to(cuda), None)
    par = torch.as_tensor(sc["parent"]).to(cuda)
    a = cast_b200.varlen_tree_attention(q, k, v, *args, parent=par)
    kpad = torch.zeros(k.shape[0], 8, 132, dtype=k.dtype, device=cuda)
    kpad[:, :, :128] = k
    k2 = kpad[:, :, :128]
    assert cast_b200.attention_plan(q, k2, v, a, 4, 128, 4196)[0] == "simt"
    b = cast_b200.varlen_tree_attention(q, k2, v, *args, parent=par)
    assert _lib.device_error() == 0
    ref = _oracle(sc, torch.bfloat16)
    assert (a.float().cpu() - ref).abs().max().item() < 2e-2
    assert (b.float().cpu() - ref).abs().max().item() < 2e-2
    assert (a.float() - b.float()).abs().max().item() < 2e-2


def _scenario(S_list, P_list, Hq=32, Hkv=8, D=128, seed=5):
    """Explicit prefix / pack lengths; random pack trees; q/k/v ~ N(0, 1)."""
    g = torch.Generator().manual_seed(seed)
    rng = np.random.default_rng(seed)
    parents = []
    for P in P_list:
        parents += [-1] + [int(rng.integers(0, i)) for i in range(1, P)]
    cu_q = np.concatenate([[0], np.cumsum(P_list)]).astype(np.int32)
    cu_kv = np.concatenate([[0], np.cumsum(np.array(S_list) + np.array(P_list))]).astype(np.int32)
    return dict(q=torch.randn(int(cu_q[-1]), Hq, D, generator=g), k=torch.randn(int(cu_kv[-1]), Hkv, D, generator=g),
                v=torch.randn(int(cu_kv[-1]), Hkv, D, generator=g), cu_q=torch.from_numpy(cu_q),
                cu_kv=torch.from_numpy(cu_kv), prefix=np.array(S_list, np.int32), pack=np.array(P_list, np.int32),
                parent=np.array(parents, np.int32))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_single_tile_ctas_two_key_streams(cuda, dtype):
    # one 128-row query tile with 2, 3, 5, 8 and 1 key tiles; a 280-row head group whose second block
    # holds one tile; a row whose only visible key is its own root (S = 0)
    sc = _scenario([200, 300, 600, 1000, 50, 500, 0], [20, 30, 7, 24, 10, 70, 3])
    got = _run(sc, dtype, cuda).float().cpu()
    err = (got - _oracle(sc, dtype)).abs().max().item()
    assert err < TOL[dtype], err


def test_single_tile_ctas_with_key_splits(cuda):
    # two long prefixes, small packs: the launch splits the keys and every chunk runs two key streams
    sc = _scenario([30000, 17001], [9, 2], seed=6)
    q16 = sc["q"].to(cuda, torch.bfloat16)
    kernel, n_split, _ = cast_b200.attention_plan(q16, sc["k"].to(cuda, torch.bfloat16),
                                                 sc["v"].to(cuda, torch.bfloat16), torch.empty_like(q16), 2, 9, 30009)
    assert kernel == "tcgen05" and n_split > 1
    got = _run(sc, torch.bfloat16, cuda).float().cpu()
    err = (got - _oracle(sc, torch.bfloat16)).abs().max().item()
    assert err < TOL[torch.bfloat16], err
