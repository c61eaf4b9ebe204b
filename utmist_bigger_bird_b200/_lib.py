"""ctypes binding of libbb_b200.so (the C ABI in include/bb_b200.h).

The library is loaded from this package directory on first use; if it is missing or cannot be
loaded, every op raises instead of falling back to another implementation.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libbb_b200.so"

BB_F16, BB_BF16, BB_F32 = 0, 1, 2
BB_POOL_MEAN, BB_POOL_MAX = 0, 1
(BB_OK, BB_ERR_ARG, BB_ERR_SHAPE, BB_ERR_DTYPE, BB_ERR_STRIDE, BB_ERR_WORKSPACE, BB_ERR_LAUNCH,
 BB_ERR_UNSUPPORTED, BB_ERR_DEVICE) = range(9)
ABI_VERSION = 2

_VALUE_ERRORS = {1, 2, 3, 4, 5, 7}
_STATUS = {0: "BB_OK", 1: "BB_ERR_ARG", 2: "BB_ERR_SHAPE", 3: "BB_ERR_DTYPE", 4: "BB_ERR_STRIDE",
           5: "BB_ERR_WORKSPACE", 6: "BB_ERR_LAUNCH", 7: "BB_ERR_UNSUPPORTED", 8: "BB_ERR_DEVICE"}

i64, f32, vp = C.c_int64, C.c_float, C.c_void_p


class RoutesArgs(C.Structure):
    _fields_ = [("q", vp), ("sq_h", i64), ("sq_t", i64),
                ("k", vp), ("sk_h", i64), ("sk_t", i64),
                ("qpos", vp),
                ("heads", i64), ("kv_heads", i64), ("n", i64), ("d", i64), ("r", i64),
                ("sink", i64), ("window", i64), ("budget", i64),
                ("scaling", f32), ("pool", C.c_int), ("dtype", C.c_int),
                ("out_idx", vp), ("so_h", i64), ("out_col", vp)]


class FlashArgs(C.Structure):
    _fields_ = [("q", vp), ("sq_h", i64), ("sq_t", i64),
                ("k", vp), ("sk_h", i64), ("sk_t", i64),
                ("v", vp), ("sv_h", i64), ("sv_t", i64),
                ("idx", vp), ("si_h", i64), ("si_g", i64), ("si_k", i64),
                ("token_mask", vp), ("sm_b", i64), ("sm_t", i64),
                ("out", vp), ("so_h", i64), ("so_t", i64),
                ("bh", i64), ("t", i64), ("n", i64), ("d", i64),
                ("num_heads", i64), ("kv_groups", i64),
                ("front", i64), ("window", i64),
                ("route_k", i64), ("route_groups", i64), ("route_chunk", i64),
                ("row_begin", i64), ("row_end", i64),
                ("scale", f32), ("dtype", C.c_int)]


class PrefillArgs(C.Structure):
    _fields_ = [("q", vp), ("sq_h", i64), ("sq_t", i64),
                ("k", vp), ("sk_h", i64), ("sk_t", i64),
                ("v", vp), ("sv_h", i64), ("sv_t", i64),
                ("cos", vp), ("sin", vp), ("sc_t", i64),
                ("qpos", vp),
                ("out", vp), ("so_h", i64), ("so_t", i64),
                ("out_idx", vp), ("si_h", i64),
                ("heads", i64), ("kv_heads", i64), ("n", i64), ("d", i64), ("r", i64),
                ("sink", i64), ("window", i64), ("budget", i64), ("exact_tail", i64),
                ("vertical_scope", i64), ("scope_chunk", i64),
                ("scaling", f32), ("pool", C.c_int), ("dtype", C.c_int)]


class EvictArgs(C.Structure):
    _fields_ = [("col", vp), ("sc_h", i64),
                ("idx", vp), ("si_h", i64), ("budget", i64),
                ("k", vp), ("sk_h", i64), ("sk_t", i64),
                ("v", vp), ("sv_h", i64), ("sv_t", i64),
                ("out_k", vp), ("sok_h", i64), ("sok_t", i64),
                ("out_v", vp), ("sov_h", i64), ("sov_t", i64),
                ("out_pos", vp),
                ("heads", i64), ("kv_heads", i64), ("n", i64), ("d", i64),
                ("sink", i64), ("window", i64), ("keep", i64), ("pool", i64), ("pool_back", i64),
                ("dtype", C.c_int)]


class DecodeArgs(C.Structure):
    _fields_ = [("q", vp), ("sq_h", i64),
                ("k", vp), ("sk_h", i64), ("sk_t", i64),
                ("v", vp), ("sv_h", i64), ("sv_t", i64),
                ("idx", vp), ("si_r", i64),
                ("route_rows", i64), ("route_k", i64),
                ("n", i64), ("n_dev", vp),
                ("cap", i64), ("heads", i64), ("kv_heads", i64), ("d", i64),
                ("front", i64), ("window", i64),
                ("scale", f32),
                ("splits", i64),
                ("out", vp), ("so_h", i64),
                ("out_probs", vp),
                ("out_idx", vp), ("so_i", i64),
                ("dtype", C.c_int), ("idx_i64", C.c_int), ("out_idx_i64", C.c_int)]


EXPORTS = {
    "bb_last_error": (C.c_char_p, []),
    "bb_abi_version": (C.c_int, []),
    "bb_kernel_launches": (C.c_uint64, []),
    "bb_device_fault": (C.c_int, [C.POINTER(C.c_int)]),
    "bb_set_wait_limit_ns": (C.c_int, [C.c_uint64]),
    "bb_debug_stall_attention": (C.c_int, [C.c_int]),
    "bb_rope_inplace": (C.c_int, [vp, C.c_int, i64, i64, i64, i64, i64, i64, i64, vp, vp, i64, i64, vp]),
    "bb_routes_workspace_size": (C.c_int, [C.POINTER(RoutesArgs), C.POINTER(C.c_size_t)]),
    "bb_routes": (C.c_int, [C.POINTER(RoutesArgs), vp, C.c_size_t, vp]),
    "bb_routes_noalloc": (C.c_int, [C.POINTER(RoutesArgs), vp]),
    "bb_flash_workspace_size": (C.c_int, [C.POINTER(FlashArgs), C.POINTER(C.c_size_t)]),
    "bb_flash": (C.c_int, [C.POINTER(FlashArgs), vp, C.c_size_t, vp]),
    "bb_sparse_prefill_workspace_size": (C.c_int, [C.POINTER(PrefillArgs), C.POINTER(C.c_size_t)]),
    "bb_sparse_prefill": (C.c_int, [C.POINTER(PrefillArgs), vp, C.c_size_t, vp]),
    "bb_kv_evict_workspace_size": (C.c_int, [C.POINTER(EvictArgs), C.POINTER(C.c_size_t)]),
    "bb_kv_evict": (C.c_int, [C.POINTER(EvictArgs), vp, C.c_size_t, vp]),
    "bb_decode_workspace_size": (C.c_int, [C.POINTER(DecodeArgs), C.POINTER(C.c_size_t)]),
    "bb_decode": (C.c_int, [C.POINTER(DecodeArgs), vp, C.c_size_t, vp]),
    "bb_decode_route_workspace_size": (C.c_int, [C.POINTER(DecodeArgs), C.POINTER(C.c_size_t)]),
    "bb_decode_route": (C.c_int, [C.POINTER(DecodeArgs), vp, C.c_size_t, vp]),
    "bb_silu_mul": (C.c_int, [vp, i64, vp, i64, i64, i64, C.c_int, vp]),
    "bb_embed_gather": (C.c_int, [vp, i64, i64, vp, i64, vp, vp, vp]),
    "bb_rmsnorm": (C.c_int, [vp, i64, vp, i64, vp, vp, i64, i64, i64, C.c_float, C.c_int, vp]),
}

_lib = None
_lock = threading.Lock()


def lib():
    """The loaded library (raises RuntimeError when it is missing: there is no fallback)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(f"{LIB_PATH.name} is not built: run `python -m utmist_bigger_bird_b200.build`")
                h = C.CDLL(str(LIB_PATH))
                for name, (res, args) in EXPORTS.items():
                    fn = getattr(h, name)
                    fn.restype = res
                    fn.argtypes = args
                if h.bb_abi_version() != ABI_VERSION:
                    raise RuntimeError(f"{LIB_PATH.name} ABI {h.bb_abi_version()} != {ABI_VERSION}")
                _lib = h
    return _lib


def check(status: int, what: str):
    if status == 0:
        return
    msg = lib().bb_last_error().decode(errors="replace")
    text = f"{what}: {msg} ({_STATUS.get(status, status)})"
    if status in _VALUE_ERRORS:
        raise ValueError(text)
    raise RuntimeError(text)
