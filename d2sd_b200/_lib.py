"""ctypes binding of the C ABI in ``include/d2sd.h`` (``libd2sd.so``).

This is the binding a maintainer of the reference would add: every entry point
takes raw pointers, element strides and sizes; no torch type crosses the
boundary. The library is loaded from the package directory (built in-tree by
``d2sd_b200.build``); there is no fallback when it is missing.
"""
from __future__ import annotations

import ctypes
import os
import threading
from ctypes import POINTER, c_float, c_int32, c_int64, c_uint64, c_void_p, c_char_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libd2sd.so"

D2SD_OK = 0
D2SD_ERR_INVALID_ARGUMENT = 1
D2SD_ERR_UNSUPPORTED = 2
D2SD_ERR_WORKSPACE = 3
D2SD_ERR_CUDA = 4
D2SD_ERR_NO_DEVICE = 5

DTYPE_F32 = 0
DTYPE_BF16 = 1
DTYPE_F16 = 2

KV_ROWS = 0
KV_UMMA_PAGES = 1

MASK_NONE = 0
MASK_CAUSAL = 1
MASK_CUSTOM = 2

SINK_NONE = 0
SINK_REFERENCE = 1
SINK_EXACT = 2

i32, i64, f32, vp = c_int32, c_int64, c_float, c_void_p
pi32 = POINTER(c_int32)

# name -> (restype, argtypes); the order of argtypes is the order in d2sd.h
SIGNATURES = {
    "d2sd_version": (i32, []),
    "d2sd_last_error": (c_char_p, []),
    "d2sd_prefix_plan_capacity": (i64, [i32, i32, i32, i32, i64]),
    "d2sd_prefix_plan": (i32, [vp, vp, vp, vp, i32, i32, i32, i32, vp, i64, vp]),
    "d2sd_partial_slot_bytes": (i64, [i32]),
    "d2sd_prefix_attention": (i32, [vp, i64, i64, i64, vp, vp, i64, i64, i64, i32, i32, i64, vp,
                                    vp, i32, i32, i32, f32, vp, i32, vp, i64, vp, vp]),
    "d2sd_suffix_merge": (i32, [vp, i64, i64, i64, vp, vp, i64, i64, i32, i32, i32, vp, vp, vp, vp,
                                vp, i64, i64, vp, i64, vp, i64, i64, vp, i64, vp, i32, i32, i32,
                                i32, i32, f32, vp, vp]),
    "d2sd_suffix_merge_gather": (i32, [vp, i64, i64, i64, vp, vp, i64, i64, i32, i32, i32, vp, vp, vp,
                                       vp, vp, i64, i64, vp, i64, vp, i64, i64, vp, i64, vp, i32,
                                       i32, i32, i32, i32, f32, vp, vp, i32, i32, i32, i64, i64,
                                       i64, vp, vp]),
    "d2sd_ipc_handle": (i32, [vp, vp, POINTER(c_int64)]),
    "d2sd_ipc_open": (i32, [vp, POINTER(c_void_p)]),
    "d2sd_ipc_close": (i32, [vp]),
    "d2sd_merge_state": (i32, [vp, i64, i64, vp, i64, vp, i64, i64, vp, i64, i64, i32, i32, i32,
                               vp]),
    "d2sd_verify_accept_workspace_size": (i64, [i32, i32, i64]),
    "d2sd_verify_accept": (i32, [vp, i32, i32, i32, i64, i64, i64, vp, i64, i64, vp, vp, vp, vp,
                                 i64, vp]),
    "d2sd_verify_accept_noalloc": (i32, [vp, i32, i32, i32, i64, i64, i64, vp, i64, i64, vp,
                                         vp, vp, vp]),
    "d2sd_verify_accept_batch_workspace_size": (i64, [i32, i32, i32, i64]),
    "d2sd_verify_accept_batch": (i32, [vp, i32, i32, i32, i32, i64, i64, i64, i64, vp, i64, i64,
                                       i64, vp, vp, vp, vp, i64, vp]),
    "d2sd_verify_accept_sharded": (i32, [vp, i32, i32, i32, i32, i64, i64, i64, i64, i64, vp,
                                         i64, i64, i64, vp, vp, vp, vp, i64, vp, vp, i32, i32,
                                         i64, vp, vp]),
    "d2sd_commit_kv_batch": (i32, [vp, i32, i32, i32, i32, i32, i32, i64, i64, i64, i64, i64,
                                   i64, i64, i32, i32, vp, vp, vp, vp, vp]),
    "d2sd_cascade_attention_f32": (i32, [vp, i64, i64, vp, vp, i64, i64, i32, i32, vp, vp, i64,
                                         i64, i32, i32, i32, vp, vp, i64, i64, vp, i64, vp, i32,
                                         vp, i64, i64, vp, i64, i32, i32, i32, f32, vp]),
    "d2sd_commit_kv": (i32, [vp, i32, i32, i32, i32, i32, i64, i64, i64, i64, i64, i64, i32, i32,
                             vp, vp, vp, i64, vp]),
    "d2sd_qk_norm_rope": (i32, [vp, i64, i64, vp, i64, i64, vp, i64, i64, vp, i64, i64, i32, i32,
                                i32, i32, i32, vp, vp, f32, vp, vp, i64, i32, vp, vp]),
    "d2sd_commit_kv_hidden": (i32, [vp, i32, i32, i32, i32, i32, i64, i64, i64, i64, i64, i64, i32,
                                    i32, vp, vp, vp, i64, vp, i32, i32, i32, i64, i64, vp, i64,
                                    vp]),
}

_lock = threading.Lock()
_lib = None


class D2SDError(RuntimeError):
    """A CUDA-side failure reported by the library."""


def load() -> ctypes.CDLL:
    """Load ``libd2sd.so`` (once). Raises if it has not been built."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `python -m d2sd_b200.build` "
                    "(there is no CPU fallback)")
            lib = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_LOCAL if hasattr(os, "RTLD_LOCAL") else 0)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def last_error() -> str:
    msg = load().d2sd_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str) -> None:
    """Turn a status code into the reference-style exception."""
    if status == D2SD_OK:
        return
    msg = f"{what}: {last_error()}"
    if status in (D2SD_ERR_INVALID_ARGUMENT, D2SD_ERR_WORKSPACE):
        raise ValueError(msg)
    if status == D2SD_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise D2SDError(msg)
