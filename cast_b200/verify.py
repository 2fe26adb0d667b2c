"""KV-cache gather of the single-sequence verify loop, on the GPU.

``gather_cache`` is cast_trees/verify.py:48-60: keep the prefix and the packed
entries listed in `keep`, in order, for every layer of a DynamicCache, in one
kernel launch (the reference runs two index_select per layer).
"""
import ctypes

import torch

from . import _lib


def cache_layers(cache):
    """(n_layers, get, put) over a DynamicCache, old and new layouts (cast_trees/verify.py:26-44)."""
    if hasattr(cache, "layers") and cache.layers and hasattr(cache.layers[0], "keys"):
        layers = cache.layers

        def get(i):
            return layers[i].keys, layers[i].values

        def put(i, k, v):
            layers[i].keys, layers[i].values = k, v
        return len(layers), get, put

    def get(i):
        return cache.key_cache[i], cache.value_cache[i]

    def put(i, k, v):
        cache.key_cache[i], cache.value_cache[i] = k, v
    return len(cache.key_cache), get, put


def gather_cache(cache, n_prefix, keep):
    """Keep the prefix and the packed entries listed in `keep`, in order (new tensors per layer)."""
    n_layers, get, put = cache_layers(cache)
    ks, vs = zip(*[get(i) for i in range(n_layers)]) if n_layers else ((), ())
    if n_layers == 0:
        return cache
    k0 = ks[0]
    if not k0.is_cuda:
        raise RuntimeError("cast_b200.gather_cache needs CUDA tensors (no CPU path)")
    for t in ks + vs:
        if t.shape != k0.shape or t.stride() != k0.stride() or t.dtype != k0.dtype or t.stride(-1) != 1:
            raise ValueError("gather_cache: every layer's K/V need one shape, one dtype and the same strides")
    dev = k0.device
    B, H, S, D = k0.shape
    keep = list(keep) if keep else []
    n_new = n_prefix + len(keep)
    keep_t = torch.tensor(keep if keep else [0], dtype=torch.int32, device=dev)
    new = [torch.empty((B, H, n_new, D), dtype=k0.dtype, device=dev) for _ in range(2 * n_layers)]
    src = []
    for k, v in zip(ks, vs):
        src += [k, v]
    P = lambda ts: (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])
    I = lambda xs: (ctypes.c_int64 * 3)(*xs)
    code = _lib.lib().cast_gather_cache(n_layers, P(src), P(new), k0.element_size(), B, H, D, S,
                                        I(k0.stride()[:3]), I(new[0].stride()[:3]), int(n_prefix),
                                        keep_t.data_ptr(), len(keep), torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(code, "cast_gather_cache")
    for i in range(n_layers):
        put(i, new[2 * i], new[2 * i + 1])
    if hasattr(cache, "_seen_tokens"):
        cache._seen_tokens = n_new
    return cache
