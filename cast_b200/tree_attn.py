"""Ragged ancestor-masked tree-verification attention on B200 (drop-in).

``varlen_tree_attention`` keeps the call signature, argument meaning and
output of cast_trees/tree_attn.py:116-139 and runs the sm_100a kernels of
``libcast_b200.so`` through its C ABI (include/cast_b200.h). Two extensions,
both keyword-only and optional:

* ``parent=``: int32 [total_q] pack-local parents (-1 for the root,
  parent[i] < i, the convention of cast_trees/serving.py:217-222). The kernel
  builds each token's ancestor bitset in shared memory, so packs are not
  limited to 64 tokens; pass ``ancestor_mask=None`` with it.
  ``ancestor_mask`` may also be int64 [total_q, W] (W words per token).
* ``max_pack=`` / ``max_kv=``: host-side bounds of pack_len and
  prefix_len + pack_len. Given, the call needs no device-to-host read; omitted,
  they are read back once, as the reference reads cu_q back (tree_attn.py:128).
* ``fp32_path=``: float32 inputs run on the tensor cores from a three-term
  bf16 split of q, k, v and the probabilities (``"split"``, the default where
  D = 128 and H_q / H_kv divides 128; within ~1e-5 of exact fp32 at
  unit-scale inputs) or on the exact CUDA-core kernel (``"exact"``).
"""
import ctypes
import math

import torch

from . import _lib

_DTYPES = {torch.float32: _lib.CAST_F32, torch.bfloat16: _lib.CAST_BF16, torch.float16: _lib.CAST_F16}


def _kernel_ready(t):
    """dim stride 1, row/head strides multiples of 4 elements, 16-byte aligned base."""
    s = t.stride()
    return s[2] == 1 and s[0] % 4 == 0 and s[1] % 4 == 0 and t.data_ptr() % 16 == 0


def _prep(t):
    return t if _kernel_ready(t) else t.contiguous()


def _i32(t, device):
    t = torch.as_tensor(t, device=device)
    return t if (t.dtype == torch.int32 and t.is_contiguous()) else t.to(torch.int32).contiguous()


def _code(dtype, D=128, G=4, fp32_path="split"):
    """C-ABI dtype code of a call: fp32 takes the split tensor-core path where it applies."""
    if dtype == torch.float32 and fp32_path == "split" and D == 128 and 128 % G == 0:
        return _lib.CAST_F32_SPLIT
    if fp32_path not in ("split", "exact"):
        raise ValueError(f"fp32_path must be 'split' or 'exact', not {fp32_path!r}")
    return _DTYPES[dtype]


def workspace_size(dtype, B, total_q, H_q, H_kv, D, max_pack, max_kv, total_kv=None, fp32_path="split"):
    code = _code(dtype, D, H_q // H_kv, fp32_path)
    if total_kv is None:
        return int(_lib.lib().cast_tree_attn_workspace_size(code, B, total_q, H_q, H_kv, D, max_pack, max_kv))
    return int(_lib.lib().cast_tree_attn_workspace_size_kv(code, B, total_q, total_kv, H_q, H_kv, D, max_pack,
                                                           max_kv))


def attention_plan(q, k, v, out, B, max_pack, max_kv, fp32_path="split"):
    """(kernel, key splits, launches) that varlen_tree_attention would use.

    kernel is "tcgen05" (tensor-core kernel), "tcgen05_split" (fp32 through the
    tensor cores from the bf16 split) or "simt" (CUDA-core kernel).
    """
    total_q, H_q, D = q.shape
    strides = (ctypes.c_int64 * 12)(*q.stride(), *k.stride(), *v.stride(), *out.stride())
    plan = (ctypes.c_int * 3)()
    code = _lib.lib().cast_tree_attn_plan(_code(q.dtype, D, H_q // k.shape[1], fp32_path), B, total_q, H_q,
                                          k.shape[1], D, max_pack, max_kv,
                                          ctypes.addressof(strides), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                          out.data_ptr(), ctypes.addressof(plan))
    _lib.check(code, "cast_tree_attn_plan")
    return {0: "simt", 1: "tcgen05", 2: "tcgen05_split"}[plan[0]], int(plan[1]), int(plan[2])


def varlen_tree_attention(q, k, v, cu_q, cu_kv, prefix_len, pack_len, ancestor_mask=None, sm_scale=None,
                          *, parent=None, max_pack=None, max_kv=None, out=None, workspace=None, fp32_path="split"):
    """q: [total_q, H_q, D], k/v: [total_kv, H_kv, D] -> [total_q, H_q, D] (q's dtype).

    cu_q / cu_kv: int32 [B+1] offsets of packs and of concat(prefix, pack).
    prefix_len / pack_len: int32 [B]. ancestor_mask: int64 [total_q] (or
    [total_q, W]); or pass parent= instead. Rows that see no key give 0.
    """
    total_q, H_q, D = q.shape
    total_kv, H_kv = k.shape[0], k.shape[1]
    assert H_q % H_kv == 0
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    if not q.is_cuda:
        raise RuntimeError("cast_b200.varlen_tree_attention needs CUDA tensors (no CPU path)")
    if q.dtype not in _DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError(f"q/k/v must share one of {list(_DTYPES)}; got {q.dtype}, {k.dtype}, {v.dtype}")
    if (ancestor_mask is None) == (parent is None):
        raise ValueError("pass exactly one of ancestor_mask and parent")
    dev = q.device
    B = int(pack_len.shape[0])
    q, k, v = _prep(q), _prep(k), _prep(v)
    if out is None:
        out = torch.empty_like(q)
    if not _kernel_ready(out):
        raise ValueError("out must have dim stride 1, row/head strides multiple of 4 and a 16-byte aligned base")
    cu_q_t, cu_kv_t = _i32(cu_q, dev), _i32(cu_kv, dev)
    prefix_t, pack_t = _i32(prefix_len, dev), _i32(pack_len, dev)
    if max_pack is None:
        max_pack = int(pack_t.max().item()) if B > 0 else 0
    if max_kv is None:
        max_kv = int((prefix_t + pack_t).max().item()) if B > 0 else 0
    anc_ptr, wpr, par_ptr = None, 0, None
    if ancestor_mask is not None:
        anc = torch.as_tensor(ancestor_mask, device=dev)
        anc = anc.to(torch.int64).reshape(total_q, -1).contiguous()
        anc_ptr, wpr = anc.data_ptr(), int(anc.shape[1])
    else:
        par = _i32(parent, dev)
        par_ptr = par.data_ptr()
    dcode = _code(q.dtype, D, H_q // H_kv, fp32_path)
    ws_bytes = int(_lib.lib().cast_tree_attn_workspace_size_kv(dcode, B, total_q, total_kv, H_q, H_kv, D,
                                                               max_pack, max_kv))
    if ws_bytes > 0 and (workspace is None or workspace.numel() * workspace.element_size() < ws_bytes
                         or workspace.data_ptr() % 256 != 0):
        workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    strides = (ctypes.c_int64 * 12)(*q.stride(), *k.stride(), *v.stride(), *out.stride())
    stream = torch.cuda.current_stream(dev).cuda_stream
    code = _lib.lib().cast_tree_attn_fwd(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), dcode, ctypes.addressof(strides),
        cu_q_t.data_ptr(), cu_kv_t.data_ptr(), prefix_t.data_ptr(), pack_t.data_ptr(),
        anc_ptr, wpr, par_ptr, B, total_q, total_kv, H_q, H_kv, D, float(sm_scale), int(max_pack), int(max_kv),
        workspace.data_ptr() if ws_bytes > 0 else None, ws_bytes, stream)
    _lib.check(code, "cast_tree_attn_fwd")
    return out


def _store_ready(t, mult):
    """dim stride 1, other strides multiples of `mult` elements (16 bytes), 16-byte aligned base."""
    st = t.stride()
    return st[-1] == 1 and all(x % mult == 0 for x in st[:-1]) and t.data_ptr() % 16 == 0


def varlen_tree_attention_store(q, k_store, v_store, k_pack, v_pack, cu_q, prefix_len, pack_len,
                                ancestor_mask=None, sm_scale=None, *, parent=None, max_pack=None, max_prefix=None,
                                out=None, workspace=None, fp32_path="split"):
    """Tree attention with each request's prefix read in place from its KV store.

    q: [total_q, H_q, D]; k_store / v_store: [B_store, H_kv, S_max, D], request
    b's prefix = rows [0, prefix_len[b]) of store row b (the per-layer stores of
    cast_trees/serving.py:190-205); k_pack / v_pack: [total_q, H_kv, D], this
    pass's keys and values in pack order (e.g. ``key[0].transpose(0, 1)`` of the
    hook's [1, H_kv, T, D] tensor, no copy). Output, masks and conventions as
    varlen_tree_attention. This replaces the hook's per-layer assembly of a
    ragged K/V copy (and its fp32 cast, cast_trees/serving.py:60-71) with the
    kernel's own addressing: prefix tiles come from the store, pack tiles from
    the pack tensors.

    16-bit inputs with D = 128 and H_q / H_kv dividing 128 run the tensor-core
    kernel directly; fp32 inputs of that shape run the split tensor-core path,
    whose split pass reads the stores in place. Other inputs are assembled into
    the ragged layout on the device (cast_kv_ragged_gather: no host read, no
    per-request loop) and run through varlen_tree_attention.
    """
    total_q, H_q, D = q.shape
    Bs, H_kv, S_max, _ = k_store.shape
    assert H_q % H_kv == 0
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    if not q.is_cuda:
        raise RuntimeError("cast_b200.varlen_tree_attention_store needs CUDA tensors (no CPU path)")
    if (ancestor_mask is None) == (parent is None):
        raise ValueError("pass exactly one of ancestor_mask and parent")
    if q.dtype not in _DTYPES or any(t.dtype != q.dtype for t in (k_store, v_store, k_pack, v_pack)):
        raise TypeError("q, the stores and the pack tensors must share one of float32, bfloat16, float16")
    dev = q.device
    B = int(pack_len.shape[0])
    cu_q_t, prefix_t, pack_t = _i32(cu_q, dev), _i32(prefix_len, dev), _i32(pack_len, dev)
    if max_pack is None:
        max_pack = int(pack_t.max().item()) if B > 0 else 0
    if max_prefix is None:
        max_prefix = int(prefix_t.max().item()) if B > 0 else 0
    G = H_q // H_kv
    code, mult = None, 8
    if D == 128 and 128 % G == 0:
        if q.dtype in (torch.bfloat16, torch.float16):
            code = _DTYPES[q.dtype]
        elif fp32_path == "split":
            code, mult = _lib.CAST_F32_SPLIT, 4
    if out is None:
        out = torch.empty_like(q)
    direct = code is not None and all(_store_ready(t, mult) for t in (q, k_store, v_store, k_pack, v_pack, out))
    L = _lib.lib()
    if not direct:
        # the ragged layout, assembled on the device, then the regular entry point
        dim1 = lambda t: t if t.stride(-1) == 1 else t.contiguous()
        k_store, v_store, k_pack, v_pack = dim1(k_store), dim1(v_store), dim1(k_pack), dim1(v_pack)
        rows_cap = B * (max_prefix + max_pack)
        k_rag = torch.empty((rows_cap, H_kv, D), dtype=q.dtype, device=dev)
        v_rag = torch.empty_like(k_rag)
        cu_kv = torch.empty(B + 1, dtype=torch.int32, device=dev)
        st14 = (ctypes.c_int64 * 14)(*k_store.stride(), *v_store.stride(), *k_pack.stride(), *v_pack.stride())
        rc = L.cast_kv_ragged_gather(k_store.data_ptr(), v_store.data_ptr(), k_pack.data_ptr(), v_pack.data_ptr(),
                                     q.element_size(), ctypes.addressof(st14), cu_q_t.data_ptr(), prefix_t.data_ptr(),
                                     pack_t.data_ptr(), B, total_q, Bs, S_max, H_kv, D, int(max_pack), rows_cap,
                                     k_rag.data_ptr(), v_rag.data_ptr(), cu_kv.data_ptr(),
                                     torch.cuda.current_stream(dev).cuda_stream)
        _lib.check(rc, "cast_kv_ragged_gather")
        res = varlen_tree_attention(q, k_rag, v_rag, cu_q_t, cu_kv, prefix_t, pack_t, ancestor_mask, sm_scale,
                                    parent=parent, max_pack=max_pack, max_kv=max_prefix + max_pack,
                                    out=out if _kernel_ready(out) else None, fp32_path=fp32_path)
        if res is not out:
            out.copy_(res)
        return out
    anc_ptr, wpr, par_ptr = None, 0, None
    if ancestor_mask is not None:
        anc = torch.as_tensor(ancestor_mask, device=dev).to(torch.int64).reshape(total_q, -1).contiguous()
        anc_ptr, wpr = anc.data_ptr(), int(anc.shape[1])
    else:
        par = _i32(parent, dev)
        par_ptr = par.data_ptr()
    ws_bytes = int(L.cast_tree_attn_store_workspace_size(code, B, total_q, H_q, H_kv, D, max_pack, max_prefix))
    if ws_bytes > 0 and (workspace is None or workspace.numel() * workspace.element_size() < ws_bytes
                         or workspace.data_ptr() % 256 != 0):
        workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    strides = (ctypes.c_int64 * 20)(*q.stride(), *k_store.stride(), *v_store.stride(), *k_pack.stride(),
                                    *v_pack.stride(), *out.stride())
    code = L.cast_tree_attn_store_fwd(
        q.data_ptr(), k_store.data_ptr(), v_store.data_ptr(), k_pack.data_ptr(), v_pack.data_ptr(), out.data_ptr(),
        code, ctypes.addressof(strides), cu_q_t.data_ptr(), prefix_t.data_ptr(), pack_t.data_ptr(),
        anc_ptr, wpr, par_ptr, B, total_q, Bs, S_max, H_q, H_kv, D, float(sm_scale), int(max_pack),
        int(max_prefix), workspace.data_ptr() if ws_bytes > 0 else None, ws_bytes,
        torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(code, "cast_tree_attn_store_fwd")
    return out
