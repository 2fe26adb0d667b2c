"""The C-ABI library without a GPU: it loads, exports every declared symbol,
and rejects bad arguments on the host before touching the device."""
import ctypes
import re

import pytest

from cast_b200 import _lib


@pytest.fixture(scope="module")
def L():
    return _lib.lib()


def test_every_declared_symbol_is_exported(L):
    decl = set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(cast_\w+)\s*\(", _lib.HEADER.read_text(), re.M))
    assert decl == set(_lib.EXPORTS)
    for name in decl:
        assert hasattr(L, name), name


def test_strerror_and_version(L):
    assert L.cast_version() == 100
    assert L.cast_strerror(0) == b"ok"
    for code in list(range(-12, 0)) + [1, 2, 4, 5]:
        assert L.cast_strerror(code) != b"unknown status"
    assert L.cast_strerror(12345) == b"unknown status"


def _attn(L, **over):
    args = dict(q=1 << 12, k=1 << 12, v=1 << 12, out=1 << 12, dtype=1, strides=None, cu_q=8, cu_kv=8,
                prefix=8, pack=8, anc=None, wpr=0, parent=8, B=1, total_q=4, total_kv=8, H_q=8, H_kv=2,
                D=128, scale=0.0, max_pack=4, max_kv=8, ws=None, ws_bytes=0, stream=None)
    args.update(over)
    strides = (ctypes.c_int64 * 12)(*([1024, 128, 1] * 4))
    if args["strides"] is None:
        args["strides"] = ctypes.addressof(strides)
    return L.cast_tree_attn_fwd(*args.values())


def test_attention_argument_checks(L):
    # every one of these returns before any CUDA call
    assert _attn(L, dtype=7) == -3
    assert _attn(L, H_q=6, H_kv=4) == -2
    assert _attn(L, D=96) == -4
    assert _attn(L, max_pack=4096) == -5
    assert _attn(L, q=None) == -1
    assert _attn(L, parent=None) == -11           # neither mask form
    assert _attn(L, anc=8, wpr=1) == -11          # both mask forms
    assert _attn(L, parent=None, anc=8, wpr=0) == -5
    bad = (ctypes.c_int64 * 12)(*([1024, 128, 2] + [1024, 128, 1] * 3))
    assert _attn(L, strides=ctypes.addressof(bad)) == -7
    assert _attn(L, q=(1 << 12) + 4) == -7
    assert _attn(L, B=0) == 0                     # empty batch is a no-op
    assert _attn(L, max_pack=0) == 0


def test_workspace_size_is_host_arithmetic(L):
    # small batch, long prefix: the key range is split and partials need scratch
    big = L.cast_tree_attn_workspace_size(1, 2, 258, 32, 8, 128, 129, 32897)
    assert big > 0 and big % 4 == 0
    # many sequences: no split, no scratch
    assert L.cast_tree_attn_workspace_size(1, 64, 8192, 32, 8, 128, 128, 8199) == 0
    assert L.cast_tree_attn_workspace_size(1, 2, 258, 30, 8, 128, 129, 32897) == 0   # bad heads


def test_fp32_split_workspace_holds_the_hi_lo_copies(L):
    # CAST_F32_SPLIT: 2 bytes of hi + 2 of lo for every element of q, k, v, plus the flags (and partials
    # when the keys are split); the size without total_kv bounds it by B * max_kv
    B, total_q, total_kv, Hq, Hkv = 64, 8192, 401408, 32, 8
    exact = L.cast_tree_attn_workspace_size_kv(3, B, total_q, total_kv, Hq, Hkv, 128, 128, 8320)
    assert exact >= 4 * 128 * (total_q * Hq + 2 * total_kv * Hkv)
    assert exact < 4 * 128 * (total_q * Hq + 2 * total_kv * Hkv) + 4096
    bound = L.cast_tree_attn_workspace_size(3, B, total_q, Hq, Hkv, 128, 128, 8320)
    assert bound >= exact
    # the other dtypes: the two size functions agree
    for dt in (0, 1, 2):
        assert (L.cast_tree_attn_workspace_size_kv(dt, 2, 258, 65794, 32, 8, 128, 129, 32897)
                == L.cast_tree_attn_workspace_size(dt, 2, 258, 32, 8, 128, 129, 32897))
    assert L.cast_tree_attn_workspace_size_kv(3, 2, 258, 100, 32, 8, 64, 129, 50) == 0     # D = 64: no split path
    # host checks of the split path: D must be 128, the workspace must be given
    assert _attn(L, dtype=3, D=64) == -4
    assert _attn(L, dtype=3) == -10 or _attn(L, dtype=3) == -6     # no device here, or no workspace


def test_tree_argument_checks(L):
    p = 1 << 12
    assert L.cast_block_topk(None, 1, 10, 10, 2, p, p, None) == -1
    assert L.cast_block_topk(p, 1, 10, 10, 0, p, p, None) == -8
    assert L.cast_block_topk(p, 1, 10, 10, 11, p, p, None) == -8
    assert L.cast_block_topk(p, 1, 10, 10, 25, p, p, None) == -8
    assert L.cast_block_topk(p, 1, 10, 5, 2, p, p, None) == -2        # row stride < V
    assert L.cast_block_topk(p, 0, 10, 10, 2, p, p, None) == 0         # no rows
    nul = None
    assert L.cast_build_tree(p, p, 1, 0, 8, 8, p, 10, p, p, p, p, p, nul, nul, nul, nul, nul, nul, None) == -2
    assert L.cast_build_tree(p, p, 1, 65, 8, 8, p, 10, p, p, p, p, p, nul, nul, nul, nul, nul, nul, None) == -2
    assert L.cast_build_tree(p, p, 1, 15, 8, 0, p, 10, p, p, p, p, p, nul, nul, nul, nul, nul, nul, None) == -8
    assert L.cast_build_tree(p, p, 1, 15, 8, 8, p, 2000, p, p, p, p, p, nul, nul, nul, nul, nul, nul, None) == -2
    # pack outputs without cu_q, pack tokens without roots
    assert L.cast_build_tree(p, p, 1, 15, 8, 8, p, 10, p, p, p, p, p, nul, p, nul, nul, nul, nul, None) == -1
    assert L.cast_build_tree(p, p, 1, 15, 8, 8, p, 10, p, p, p, p, p, p, nul, nul, p, nul, nul, None) == -1
    assert L.cast_build_tree(p, p, 0, 15, 8, 8, p, 10, p, p, p, p, p, nul, nul, nul, nul, nul, nul, None) == 0


def test_walk_select_append_gather_argument_checks(L):
    # argument errors come back before any CUDA call
    p = 1 << 12
    walk = lambda **o: L.cast_tree_walk_greedy(*dict(dict(
        logits=p, dtype=1, row_stride=64, V=64, cu_q=p, par=p, tok=p, B=2, total_q=8, cap=4, path=p, acc=p,
        bonus=p, keep=None, tokens=None, stream=None), **o).values())
    assert walk(dtype=9) == -3
    assert walk(V=0) == -2 and walk(row_stride=32) == -2 and walk(cap=0) == -2
    assert walk(logits=None) == -1 and walk(bonus=None) == -1
    assert walk(B=0) == 0
    sel = lambda **o: L.cast_select_global_topk(*dict(dict(
        tok=p, dep=p, par=p, sc=p, cnt=p, B=4, mb=48, total=16, otok=p * 2, odep=p * 2, opar=p * 2, osc=p * 2,
        ocnt=p * 2, cu_q=None, rt=None, sl=None, pp=None, pt=None, ppos=None, cap=0, stream=None), **o).values())
    assert sel(mb=0) == -2 and sel(mb=2048) == -2 and sel(B=100000) == -2
    assert sel(tok=None) == -1 and sel(ocnt=None) == -1
    assert sel(pp=p) == -1                        # pack arrays need cu_q
    assert sel(cu_q=p, pt=p) == -1                # pack tokens need root tokens
    assert sel(otok=p) == -7                      # outputs may not be the inputs
    assert sel(B=0) == 0
    ptrs = (ctypes.c_void_p * 2)(p, p)
    st = (ctypes.c_int64 * 3)(1024, 128, 1)
    app = lambda **o: L.cast_append_store(*dict(dict(
        L=1, src=ptrs, dst=ptrs, pack=ptrs, es=2, H=8, D=128, Bs=2, scap=16, sst=st, Bd=2, dcap=16, dst_st=st,
        prow=8, pst=st, rows=None, sl=p, acc=p, keep=p, ks=4, cu=p, app=1, stream=None), **o).values())
    assert app(es=3) == -3
    assert app(H=0) == -2 and app(Bd=40000) == -2
    assert app(keep=None) == -1
    assert app(rows=p) == -2                      # append in place takes no row map
    other = (ctypes.c_void_p * 2)(p * 2, p * 2)
    assert app(dst=other) == -2                   # ... and writes the stores it reads
    assert app(L=0) == 0 and app(Bd=0) == 0
    gat = lambda **o: L.cast_gather_cache(*dict(dict(
        L=1, src=ptrs, dst=other, es=2, B=1, H=8, D=128, slen=20, sst=st, dst_st=st, npre=12, keep=p, nk=3,
        stream=None), **o).values())
    assert gat(es=8) == -3
    assert gat(npre=30) == -2 and gat(nk=-1) == -2
    assert gat(keep=None) == -1
    assert gat(B=0) == 0 and gat(npre=0, nk=0) == 0
