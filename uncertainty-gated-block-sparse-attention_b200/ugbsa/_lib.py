"""ctypes binding of libugbsa.so (the C ABI declared in include/ugbsa.h).

This is the only way the Python package reaches the GPU: there is no CPU or
PyTorch fallback.  If the shared object is missing or fails to load, every op
raises ``RuntimeError``.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
# UGBSA_LIB overrides the location (another build of the same library, e.g. to compare two builds)
LIB_PATH = os.environ.get("UGBSA_LIB") or os.path.join(_HERE, "_lib", "libugbsa.so")

UGBSA_OK = 0
F32, BF16, F16 = 0, 1, 2
MODE = {"topk": 0, "quest": 1, "router": 2}
SCORE = {"mean": 0, "quest": 1}
ROUTER_MODE = {"abs": 0, "quantile": 1}
GRAIN = {"cell": 0, "row": 1}
NORM_SCALE, NORM_OFFSET, NORM_NONE = 0, 1, 2


class Strides(ctypes.Structure):
    """ugbsa_strides: element strides of a [B, H, S, D] view."""
    _fields_ = [("b", ctypes.c_int64), ("h", ctypes.c_int64), ("s", ctypes.c_int64), ("d", ctypes.c_int64)]


class SelectorConfig(ctypes.Structure):
    """ugbsa_selector_config: the Selector knobs of the v2 path."""
    _fields_ = [("mode", ctypes.c_int), ("router_score", ctypes.c_int), ("router_mode", ctypes.c_int),
                ("router_grain", ctypes.c_int), ("router_quantile", ctypes.c_double),
                ("router_tau", ctypes.c_double), ("budget_blocks", ctypes.c_int), ("k_min", ctypes.c_int),
                ("k_max", ctypes.c_int)]


class IpcHandle(ctypes.Structure):
    """ugbsa_ipc_handle: opaque 64-byte handle of a peer-mappable device buffer."""
    _fields_ = [("bytes", ctypes.c_ubyte * 64)]


# name -> (restype, argtypes); mirrors include/ugbsa.h
P = ctypes.c_void_p
I = ctypes.c_int
SIGNATURES = {
    "ugbsa_version": (I, []),
    "ugbsa_status_string": (ctypes.c_char_p, [I]),
    "ugbsa_select_budget": (I, [ctypes.POINTER(SelectorConfig), I, ctypes.POINTER(I), ctypes.POINTER(I)]),
    "ugbsa_select_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(SelectorConfig), I, I, I]),
    "ugbsa_select_workspace_bytes_ex": (ctypes.c_size_t, [ctypes.POINTER(SelectorConfig), I, I, I, I, I, I]),
    "ugbsa_block_summary": (I, [P, I, Strides, I, I, I, I, I, P, P, P, P]),
    "ugbsa_select": (I, [P, I, Strides, P, P, I, I, I, I, I, ctypes.c_float, ctypes.POINTER(SelectorConfig),
                         P, I, P, P, P, ctypes.c_size_t, P]),
    "ugbsa_select_noalloc": (I, [P, I, Strides, P, P, I, I, I, I, I, ctypes.c_float,
                                 ctypes.POINTER(SelectorConfig), P, I, P, P, P]),
    "ugbsa_select_tiles": (I, [P, I, Strides, P, P, I, I, I, I, I, ctypes.c_float,
                               ctypes.POINTER(SelectorConfig), P, I, P, P, P, ctypes.c_size_t, P]),
    "ugbsa_select_finish_workspace_bytes": (ctypes.c_size_t, [I, I]),
    "ugbsa_select_finish": (I, [P, P, I, I, I, I, ctypes.POINTER(SelectorConfig), P, I, P, P, P, ctypes.c_size_t,
                                P]),
    "ugbsa_attn": (I, [P, P, P, I, Strides, Strides, Strides, P, I, I, I, I, I, I, I, ctypes.c_float, P,
                       Strides, P]),
    "ugbsa_read_device_error": (I, [P, ctypes.POINTER(I)]),
    "ugbsa_check_wait_limit": (I, [P]),
    "ugbsa_check_bf16_fma": (I, [P, P, P, P, P, I, P]),
    "ugbsa_select_tiles_rows": (I, [P, I, Strides, P, P, I, I, I, I, I, I, I, I, ctypes.c_float,
                                    ctypes.POINTER(SelectorConfig), P, I, P, P, P, ctypes.c_size_t, P]),
    "ugbsa_select_finish_rows": (I, [P, P, I, I, I, I, I, I, I, ctypes.POINTER(SelectorConfig), P, I, P, P, P,
                                     ctypes.c_size_t, P]),
    "ugbsa_attn_rows": (I, [P, P, P, I, Strides, Strides, Strides, P, I, I, I, I, I, I, I, I, I, ctypes.c_float, P,
                            Strides, P]),
    "ugbsa_attn_rows_peers": (I, [P, P, P, I, Strides, Strides, Strides, P, I, I, I, I, I, I, I, I, I,
                                  ctypes.c_float,
                                  P, Strides, ctypes.POINTER(P), I, P]),
    "ugbsa_peer_buffer_alloc": (I, [ctypes.c_size_t, ctypes.POINTER(P), ctypes.POINTER(IpcHandle)]),
    "ugbsa_peer_buffer_open": (I, [ctypes.POINTER(IpcHandle), ctypes.POINTER(P)]),
    "ugbsa_peer_buffer_close": (I, [P]),
    "ugbsa_peer_buffer_free": (I, [P]),
    "ugbsa_block_summary_update": (I, [P, I, Strides, I, I, I, I, I, I, I, P, P, P]),
    "ugbsa_decode_workspace_bytes": (ctypes.c_size_t, [I, I, I, I, I]),
    "ugbsa_decode_select": (I, [P, I, Strides, P, P, I, I, I, I, I, I, ctypes.c_float,
                                ctypes.POINTER(SelectorConfig), P, I, P, P, P, ctypes.c_size_t, P]),
    "ugbsa_decode_attn": (I, [P, P, P, I, Strides, Strides, Strides, P, I, I, I, I, I, I, ctypes.c_float, P, Strides,
                              P, ctypes.c_size_t, P]),
    "ugbsa_decode_step": (I, [P, P, P, I, Strides, Strides, Strides, P, P, I, I, I, I, I, I, ctypes.c_float,
                              ctypes.POINTER(SelectorConfig), P, I, P, P, P, Strides, P, ctypes.c_size_t, P]),
    "ugbsa_qk_norm_rope": (I, [P, I, Strides, P, I, ctypes.c_float, P, P, ctypes.c_int64, ctypes.c_int64, I, I, I,
                               I, I, P, Strides, I, P, P, P]),
    "ugbsa_select_rows_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(SelectorConfig), I, I, I]),
    "ugbsa_select_rows": (I, [P, I, Strides, P, P, I, I, I, I, I, ctypes.c_float, ctypes.POINTER(SelectorConfig),
                              P, P, P, P, P, ctypes.c_size_t, P]),
    "ugbsa_keep_to_tiles": (I, [P, P, I, I, I, P, P]),
    "ugbsa_attn_rowmask": (I, [P, P, P, I, Strides, Strides, Strides, P, I, P, I, I, I, I, I, ctypes.c_float, P,
                               Strides, P]),
    "ugbsa_block_order_stats_workspace_bytes": (ctypes.c_size_t, [I, I, I]),
    "ugbsa_block_order_stats": (I, [P, I, Strides, P, P, I, I, I, I, I, ctypes.c_float, I, I, P, P, P, P, P, P,
                                    ctypes.c_size_t, P]),
}

_lib = None
_lock = threading.Lock()


def load():
    """Load libugbsa.so (raises RuntimeError if it is missing: no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"libugbsa.so not found at {LIB_PATH}; build it with `python -m ugbsa._build` "
                "(nvcc, sm_100a). There is no CPU fallback.")
        try:
            import torch  # noqa: F401  (loads the CUDA runtime the library links against)
        except ImportError:
            pass
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def status_string(rc: int) -> str:
    return load().ugbsa_status_string(rc).decode()


def check(rc: int, what: str) -> None:
    if rc != UGBSA_OK:
        raise RuntimeError(f"{what} failed: {status_string(rc)} (status {rc})")
