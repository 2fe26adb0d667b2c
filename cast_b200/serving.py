"""KV-store append / compaction of the batched verify loop, on the GPU.

``append_store`` is cast_trees/serving.py:264-289 (BatchedServer._append_store)
as a function: after the walk, the accepted pack K/V rows of every surviving
request are appended to its per-layer store, finished requests are dropped
(the stores are compacted) and the capacity grows when needed, with the
reference's shapes and zero-filled tails. One kernel launch covers every
layer (the reference issues two gathers and two scatters per layer).

``append_store_inplace`` is the all-device form for rounds where no request
leaves and no store grows: keep / accepted come straight from the walk's
device output and only the appended rows are written.
"""
import ctypes

import numpy as np
import torch

from . import _lib


def _ptrs(tensors):
    return (ctypes.c_void_p * len(tensors))(*[t.data_ptr() for t in tensors])


def _i64(*xs):
    return (ctypes.c_int64 * len(xs))(*xs)


def _pairs(ks, vs):
    out = []
    for k, v in zip(ks, vs):
        out += [k, v]
    return out


def _check_layers(bufs, what):
    shape, stride = bufs[0].shape, bufs[0].stride()
    for t in bufs:
        if not t.is_cuda:
            raise RuntimeError(f"cast_b200 {what} needs CUDA tensors (no CPU path)")
        if t.shape != shape or t.stride() != stride or t.dtype != bufs[0].dtype or t.stride(-1) != 1:
            raise ValueError(f"{what}: every layer's tensors need one shape, one dtype and the same strides")


def append_store(buf_k, buf_v, store_len, cu_q, keep, accepted, rows, pack_k, pack_v):
    """Append the accepted pack K/V of surviving requests, drop the rest.

    buf_k / buf_v: per-layer stores [B, H, cap, D]; store_len, cu_q, accepted:
    host ints per request (cu_q: pack offsets of the verify pass); keep: per
    request the pack-local rows to append ([0] + [i + 1 for i in path]); rows:
    surviving requests; pack_k / pack_v: per-layer pass K/V [H, total_q, D]
    (the hook's key[0] / value[0]). Returns (buf_k, buf_v, new_len) exactly as
    the reference: the same tensors appended in place when no request leaves
    and no store grows, else new stores (whole store rows gathered in `rows`
    order, capacity max(max(new_len), 2 * cap) when it grows with the new
    rows zero, then the appended rows written).
    """
    L = len(buf_k)
    new_len = [store_len[b] + accepted[b] for b in rows]
    _check_layers(list(buf_k) + list(buf_v), "append_store")
    _check_layers(list(pack_k) + list(pack_v), "append_store pack")
    dev = buf_k[0].device
    B_src, H, cap, D = buf_k[0].shape
    compact = len(rows) != len(store_len)
    new_cap = cap
    if max(new_len) > cap:
        new_cap = max(max(new_len), 2 * cap)
    in_place = not compact and new_cap == cap
    ks = max(1, max((len(keep[b]) for b in range(len(keep))), default=1))
    n_keep = [len(keep[b]) for b in range(B_src)]
    keep_arr = np.full((B_src, ks), -1, dtype=np.int32)
    for b in range(B_src):
        keep_arr[b, :n_keep[b]] = keep[b]
    meta = np.concatenate([np.asarray(store_len[:B_src], np.int32), np.asarray(n_keep, np.int32),
                           np.asarray(cu_q[:B_src], np.int32), np.asarray(rows, np.int32),
                           keep_arr.reshape(-1)])
    m = torch.from_numpy(meta).to(dev)
    sl, acc, cq = m[:B_src], m[B_src:2 * B_src], m[2 * B_src:3 * B_src]
    rw = m[3 * B_src:3 * B_src + len(rows)]
    kp = m[3 * B_src + len(rows):]
    if in_place:
        new_k, new_v = list(buf_k), list(buf_v)
    else:
        mk = lambda: torch.empty((len(rows), H, new_cap, D), dtype=buf_k[0].dtype, device=dev)
        new_k = [mk() for _ in range(L)]
        new_v = [mk() for _ in range(L)]
    src = _pairs(buf_k, buf_v)
    dst = _pairs(new_k, new_v)
    pk = _pairs(pack_k, pack_v)
    p0 = pack_k[0]
    code = _lib.lib().cast_append_store(
        L, _ptrs(src), _ptrs(dst), _ptrs(pk), buf_k[0].element_size(), H, D, B_src, cap,
        _i64(*buf_k[0].stride()[:3]), len(rows), new_cap, _i64(*dst[0].stride()[:3]), p0.shape[1],
        _i64(0, p0.stride(0), p0.stride(1)), None if in_place else rw.data_ptr(), sl.data_ptr(), acc.data_ptr(),
        kp.data_ptr(), ks, cq.data_ptr(), 1 if in_place else 0, torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(code, "cast_append_store")
    return new_k, new_v, new_len


def append_store_inplace(buf_k, buf_v, store_len, cu_q, keep, accepted, pack_k, pack_v):
    """Append in place from device metadata (no request leaves, no store grows).

    store_len / cu_q / accepted: int32 [B] CUDA tensors; keep: int32 [B, w]
    CUDA tensor (a Walk's keep rows). The caller guarantees
    store_len + accepted <= cap (violations are skipped and recorded as a
    device error). Returns nothing; the new lengths are store_len + accepted.
    """
    L = len(buf_k)
    _check_layers(list(buf_k) + list(buf_v), "append_store_inplace")
    _check_layers(list(pack_k) + list(pack_v), "append_store_inplace pack")
    dev = buf_k[0].device
    B, H, cap, D = buf_k[0].shape
    i32 = lambda t: torch.as_tensor(t, device=dev).to(torch.int32).contiguous()
    sl, cq, acc, kp = i32(store_len), i32(cu_q), i32(accepted), i32(keep)
    if kp.dim() != 2 or kp.shape[0] != B or sl.numel() != B or cq.numel() < B or acc.numel() != B:
        raise ValueError("append_store_inplace: store_len / cu_q / accepted need B entries and keep [B, w]")
    src = _pairs(buf_k, buf_v)
    p0 = pack_k[0]
    st = _i64(*buf_k[0].stride()[:3])
    code = _lib.lib().cast_append_store(
        L, _ptrs(src), _ptrs(src), _ptrs(_pairs(pack_k, pack_v)), buf_k[0].element_size(), H, D, B, cap, st,
        B, cap, st, p0.shape[1], _i64(0, p0.stride(0), p0.stride(1)), None, sl.data_ptr(), acc.data_ptr(),
        kp.data_ptr(), kp.shape[1], cq.data_ptr(), 1, torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(code, "cast_append_store")
