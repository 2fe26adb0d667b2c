"""Loader and build recipe of the in-tree C-ABI library ``libcast_b200.so``.

The library is built by nvcc straight from ``cast_b200/csrc`` for sm_100a
(``build()``) and loaded with ctypes. There is no CPU fallback: every entry
point in this package raises if the library or a CUDA device is missing.
"""
import ctypes
import os
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB_PATH = Path(os.environ["CAST_B200_LIB"]) if os.environ.get("CAST_B200_LIB") else PKG / "libcast_b200.so"
HEADER = ROOT / "include" / "cast_b200.h"

NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
              "-Xcompiler", "-fPIC", "-shared"]

# status codes of include/cast_b200.h
CAST_OK = 0
CAST_F32, CAST_BF16, CAST_F16, CAST_F32_SPLIT = 0, 1, 2, 3
CAST_MAX_PACK = 1024
CAST_MAX_TOPK = 24
CAST_MAX_DEPTH = 64
CAST_DEV_BAD_LAYOUT, CAST_DEV_BAD_PARENT, CAST_DEV_TIMEOUT, CAST_DEV_TREE_OVERFLOW = 1, 2, 4, 5

# every symbol include/cast_b200.h declares
EXPORTS = ("cast_strerror", "cast_version", "cast_device_error", "cast_tree_attn_fwd",
           "cast_tree_attn_workspace_size", "cast_tree_attn_plan", "cast_block_topk", "cast_build_tree",
           "cast_tree_attn_fwd_noalloc", "cast_tree_attn_store_fwd", "cast_tree_attn_store_workspace_size",
           "cast_tree_walk_greedy", "cast_select_global_topk", "cast_append_store", "cast_gather_cache",
           "cast_test_set_wait_limit_ns", "cast_tree_attn_workspace_size_kv", "cast_kv_ragged_gather",
           "cast_test_set_tc_kernel")
CAST_NOALLOC_SCRATCH_BYTES = 64 << 20


def _sources():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [HEADER]


def needs_build():
    if os.environ.get("CAST_B200_LIB"):
        return False          # an explicitly chosen build is used as it is
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    return any(s.stat().st_mtime > t for s in _sources())


def build(force=False, verbose=False):
    """Compile csrc/capi.cu (which includes every kernel) into libcast_b200.so."""
    if not force and not needs_build():
        return LIB_PATH
    nvcc = os.environ.get("NVCC", "nvcc")
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, *NVCC_FLAGS, "-o", str(tmp), str(CSRC / "capi.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    if verbose:
        print(res.stderr)
    return LIB_PATH


_LIB = None


def lib():
    """The loaded library with argument types declared (builds it if stale)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if needs_build():
        build()
    L = ctypes.CDLL(str(LIB_PATH))
    c_int, c_i64, c_vp, c_sz = ctypes.c_int, ctypes.c_int64, ctypes.c_void_p, ctypes.c_size_t
    L.cast_strerror.restype = ctypes.c_char_p
    L.cast_strerror.argtypes = [c_int]
    L.cast_version.restype = c_int
    L.cast_version.argtypes = []
    L.cast_device_error.restype = c_int
    L.cast_device_error.argtypes = [c_vp]
    L.cast_tree_attn_fwd.restype = c_int
    L.cast_tree_attn_fwd.argtypes = [c_vp, c_vp, c_vp, c_vp, c_int, c_vp,
                                     c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_vp,
                                     c_int, c_int, c_int, c_int, c_int, c_int,
                                     ctypes.c_float, c_int, c_int, c_vp, c_sz, c_vp]
    L.cast_tree_attn_fwd_noalloc.restype = c_int
    L.cast_tree_attn_fwd_noalloc.argtypes = [c_vp, c_vp, c_vp, c_vp, c_int, c_vp,
                                             c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_vp,
                                             c_int, c_int, c_int, c_int, c_int, c_int,
                                             ctypes.c_float, c_int, c_int, c_vp]
    L.cast_tree_attn_store_fwd.restype = c_int
    L.cast_tree_attn_store_fwd.argtypes = [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_vp,
                                           c_vp, c_vp, c_vp, c_vp, c_int, c_vp,
                                           c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                           ctypes.c_float, c_int, c_int, c_vp, c_sz, c_vp]
    L.cast_tree_attn_store_workspace_size.restype = c_sz
    L.cast_tree_attn_store_workspace_size.argtypes = [c_int] * 8
    L.cast_tree_attn_plan.restype = c_int
    L.cast_tree_attn_plan.argtypes = [c_int] * 8 + [c_vp] * 6
    L.cast_tree_attn_workspace_size.restype = c_sz
    L.cast_tree_attn_workspace_size.argtypes = [c_int] * 8
    L.cast_kv_ragged_gather.restype = c_int
    L.cast_kv_ragged_gather.argtypes = [c_vp, c_vp, c_vp, c_vp, c_int, c_vp, c_vp, c_vp, c_vp,
                                        c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_i64, c_vp, c_vp, c_vp,
                                        c_vp]
    L.cast_tree_attn_workspace_size_kv.restype = c_sz
    L.cast_tree_attn_workspace_size_kv.argtypes = [c_int] * 9
    L.cast_block_topk.restype = c_int
    L.cast_block_topk.argtypes = [c_vp, c_i64, c_i64, c_i64, c_int, c_vp, c_vp, c_vp]
    L.cast_build_tree.restype = c_int
    L.cast_build_tree.argtypes = [c_vp, c_vp, c_int, c_int, c_int, c_int, c_vp, c_int,
                                  c_vp, c_vp, c_vp, c_vp, c_vp,
                                  c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp]
    L.cast_tree_walk_greedy.restype = c_int
    L.cast_tree_walk_greedy.argtypes = [c_vp, c_int, c_i64, c_int, c_vp, c_vp, c_vp, c_int, c_int, c_int,
                                        c_vp, c_vp, c_vp, c_vp, c_vp, c_vp]
    L.cast_select_global_topk.restype = c_int
    L.cast_select_global_topk.argtypes = [c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_i64,
                                          c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                          c_vp, c_vp, c_vp, c_i64, c_vp]
    L.cast_append_store.restype = c_int
    L.cast_append_store.argtypes = [c_int, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_i64, c_vp,
                                    c_int, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_vp,
                                    c_int, c_vp]
    L.cast_gather_cache.restype = c_int
    L.cast_gather_cache.argtypes = [c_int, c_vp, c_vp, c_int, c_int, c_int, c_int, c_i64, c_vp, c_vp, c_int,
                                    c_vp, c_int, c_vp]
    L.cast_test_set_wait_limit_ns.restype = None
    L.cast_test_set_wait_limit_ns.argtypes = [ctypes.c_uint64]
    L.cast_test_set_tc_kernel.restype = None
    L.cast_test_set_tc_kernel.argtypes = [c_int]
    _LIB = L
    return L


class CastError(RuntimeError):
    """A status code returned by the C ABI."""

    def __init__(self, code, where):
        self.code = code
        msg = lib().cast_strerror(code).decode()
        super().__init__(f"{where}: {msg} (status {code})")


def check(code, where):
    if code != CAST_OK:
        raise CastError(code, where)


def device_error(stream=None):
    """Reads and clears the device error word (synchronises the stream)."""
    import torch
    st = torch.cuda.current_stream() if stream is None else stream
    return lib().cast_device_error(ctypes.c_void_p(st.cuda_stream))


def raise_device_error(where, stream=None):
    code = device_error(stream)
    if code != CAST_OK:
        raise CastError(code, where)
