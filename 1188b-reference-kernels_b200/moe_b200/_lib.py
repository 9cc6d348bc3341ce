"""ctypes binding of ``libmoe_b200.so`` (the C ABI in ``include/moe_b200.h``).

This is the only place that touches the shared library. There is no fallback:
if the library is missing or fails to load, every op raises.
"""
from __future__ import annotations

import ctypes
import threading
from ctypes import c_char_p, c_int32, c_int64, c_size_t, c_void_p, POINTER

from . import build as _build

MOE_OK = 0
MOE_ERR_INVALID = 1
MOE_ERR_UNSUPPORTED = 2
MOE_ERR_CUDA = 3
MOE_ERR_DEVICE = 4

_STATUS_NAMES = {
    MOE_ERR_INVALID: "invalid argument",
    MOE_ERR_UNSUPPORTED: "unsupported",
    MOE_ERR_CUDA: "CUDA error",
    MOE_ERR_DEVICE: "device error",
}


class MoeError(RuntimeError):
    """A C-ABI call returned a non-zero moe_status."""

    def __init__(self, func: str, status: int, message: str):
        self.func = func
        self.status = status
        super().__init__(f"{func}: {_STATUS_NAMES.get(status, status)}: {message}")


# name -> argtypes; every function returns int (moe_status) unless listed in _RESTYPE.
_SIGNATURES = {
    "moe_b200_last_error": [],
    "moe_b200_abi_version": [],
    "moe_topk_f32": [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int32, c_void_p],
    "moe_router_topk": [c_void_p, c_void_p, c_int64, c_int64, c_int32, c_int32, c_int32,
                        c_void_p, c_void_p, c_void_p, c_void_p, c_void_p],
    "moe_router_topk_placed": [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int32, c_int32,
                               c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p],
    "moe_router_gemm_topk": [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int32,
                             c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                             c_void_p, c_void_p],
    "moe_row_id_map_workspace_size": [c_int64, c_int64, POINTER(c_size_t)],
    "moe_row_id_map": [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                       c_void_p, c_void_p, c_size_t, c_void_p],
    "moe_row_id_map_static_scratch": [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p,
                                      c_void_p, c_void_p, c_void_p],
    "moe_permute_mask_map": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64,
                             c_int64, c_int64, c_void_p],
    "moe_permute_mask_map_trans": [c_void_p, c_void_p, c_int32, c_void_p, c_void_p, c_void_p,
                                   c_int64, c_int64, c_int64, c_int64, c_void_p],
    "moe_unpermute_mask": [c_void_p, c_void_p, c_int32, c_void_p, c_int32, c_void_p, c_void_p,
                           c_int64, c_int64, c_int64, c_int64, c_void_p],
    "moe_unpermute_mask_token_major": [c_void_p, c_void_p, c_void_p, c_int32, c_void_p,
                                       c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p],
    "moe_permute_backward": [c_void_p, c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_void_p,
                             c_int64, c_int64, c_int64, c_int64, c_void_p],
    "moe_combine_backward": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                             c_int64, c_int64, c_int64, c_int64, c_void_p],
    "moe_swiglu_backward": [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p],
    "moe_grouped_gemm_workspace_size": [c_int64, POINTER(c_size_t)],
    "moe_grouped_gemm_plan_splits": [c_void_p, c_int64, c_int64, c_void_p, c_size_t, c_void_p],
    "moe_grouped_gemm_plan_ep": [c_void_p, c_int64, c_int64, c_void_p, c_size_t, c_void_p],
    "moe_grouped_gemm": [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64,
                         c_int64, c_int32, c_void_p, c_size_t, c_void_p],
    "moe_ep_dispatch_dedup": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                              c_void_p, c_int32, c_int32, c_int32, c_int64, c_int64, c_int64,
                              c_int64, c_int64, c_void_p],
    "moe_ep_expand": [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int64,
                      c_int64, c_int64, c_void_p],
    "moe_grouped_wgrad_workspace_size": [c_int64, POINTER(c_size_t)],
    "moe_grouped_wgrad": [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64,
                          c_void_p, c_void_p, c_size_t, c_void_p],
    "moe_grouped_wgrad_dev": [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64,
                              c_void_p, c_void_p, c_size_t, c_void_p],
    "moe_grouped_gemm_nn": [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64,
                         c_int64, c_int32, c_void_p, c_size_t, c_void_p],
    "moe_grouped_gemm_check": [c_void_p, c_size_t, c_void_p, POINTER(c_int32)],
    "moe_swiglu": [c_void_p, c_void_p, c_int64, c_int64, c_void_p],
    "moe_ipc_get_handle": [c_void_p, c_void_p, POINTER(ctypes.c_uint64)],
    "moe_ipc_open_handle": [c_void_p, POINTER(c_void_p)],
    "moe_ipc_close_handle": [c_void_p],
    "moe_copy_async": [c_void_p, c_void_p, c_size_t, c_void_p],
    "moe_ep_dispatch": [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int64,
                        c_int64, c_int64, c_int64, c_int64, c_void_p],
    "moe_permute_check": [c_void_p, POINTER(c_int32)],
    "moe_permute_topk": [c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_void_p, c_void_p,
                         c_int64, c_int64, c_int64, c_int64, c_void_p],
    "moe_ep_pull_stage": [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p,
                          c_void_p, c_void_p],
    "moe_ep_dispatch_pull": [c_void_p, c_void_p, c_int32, c_int64, c_int64, c_void_p, c_int32,
                             c_void_p, c_int64, c_int64, c_int64, c_void_p],
    "moe_ep_combine_backward": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                c_int32, c_int32, c_int64, c_void_p, c_int64, c_int64, c_int64,
                                c_int64, c_void_p],
    "moe_ep_dispatch_range": [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32,
                              c_int64, c_int64, c_int64, c_int64, c_int64, c_int32, c_int32,
                              c_int32, c_void_p],
    "moe_ep_combine": [c_void_p, c_void_p, c_int32, c_int32, c_int64, c_void_p, c_void_p,
                       c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p],
}
_RESTYPE = {"moe_b200_last_error": c_char_p}

EXPORTED = tuple(_SIGNATURES)

# Kernels each successful call launches (for the bench's launch count). A
# grouped GEMM is two launches on B200: the CTA-pair kernel on whole 256-row
# tiles, then the single-CTA kernel on the group remainders (one launch only
# when CTA pairs are disabled with MOE_GEMM_PAIR=0 or MOE_GEMM_SPLIT=0).
_LAUNCHES = {"moe_topk_f32": 1, "moe_router_topk": 1, "moe_router_topk_placed": 1,
             "moe_router_gemm_topk": 1,
             "moe_row_id_map": 3,
             "moe_row_id_map_static_scratch": 3,
             "moe_permute_mask_map": 1, "moe_permute_mask_map_trans": 1, "moe_unpermute_mask": 1,
             "moe_unpermute_mask_token_major": 1, "moe_ep_dispatch": 1, "moe_ep_combine": 1,
             "moe_ep_dispatch_range": 1, "moe_ep_combine_backward": 1,
             "moe_ep_pull_stage": 1, "moe_ep_dispatch_pull": 1, "moe_permute_topk": 1,
             "moe_permute_backward": 1, "moe_ep_dispatch_dedup": 1, "moe_ep_expand": 1,
             "moe_combine_backward": 1, "moe_swiglu_backward": 1,
             "moe_grouped_gemm_plan_splits": 1, "moe_grouped_gemm_plan_ep": 1,
             "moe_grouped_gemm": 2, "moe_grouped_gemm_nn": 2, "moe_grouped_wgrad": 3,
             "moe_grouped_wgrad_dev": 3,
             "moe_swiglu": 1}
launch_count = 0

_lock = threading.Lock()
_lib = None


def load(path=None, build_if_missing: bool = False):
    """Loads (once) and returns the ctypes handle of libmoe_b200.so."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = path or _build.LIB_PATH
        if not p.exists():
            if build_if_missing:
                _build.build()
            else:
                raise ImportError(
                    f"{p} is missing: build it with `python {_build.__file__}` "
                    "(the MoE B200 ops have no CPU fallback)")
        lib = ctypes.CDLL(str(p))
        for name, args in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = _RESTYPE.get(name, c_int32)
        if lib.moe_b200_abi_version() != 2:
            raise ImportError("libmoe_b200.so ABI version mismatch")
        _lib = lib
        return _lib


def call(name: str, *args) -> None:
    """Calls a C-ABI function and raises MoeError on a non-zero status."""
    global launch_count
    lib = load()
    st = getattr(lib, name)(*args)
    if st != MOE_OK:
        msg = lib.moe_b200_last_error().decode(errors="replace")
        raise MoeError(name, st, msg)
    launch_count += _LAUNCHES.get(name, 0)


def last_error() -> str:
    return load().moe_b200_last_error().decode(errors="replace")
