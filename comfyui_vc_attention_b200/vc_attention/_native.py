"""ctypes binding of libvcattn.so (the C ABI declared in include/vcattn.h).

The library is built in-tree by ``comfyui_vc_attention_b200.build``.  Loading
is lazy and loud: ``lib()`` raises ``NativeUnavailable`` with the reason when
the shared object is missing or fails to load; nothing here substitutes a CPU
implementation.
"""

from __future__ import annotations

import ctypes
import os
import threading
from ctypes import (POINTER, Structure, c_char_p, c_double, c_float, c_int, c_int64, c_size_t,
                    c_uint8, c_void_p)
from typing import Optional

_PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.environ.get("VCATTN_LIB", os.path.join(_PKG, "libvcattn.so"))
HEADER_PATH = os.path.join(os.path.dirname(_PKG), "include", "vcattn.h")

OK = 0
ERR_ARG = 1
ERR_CUDA = 2
ERR_WORKSPACE = 3
ERR_DEVICE = 4
ERR_INJECTED = 5

DTYPE_BF16 = 0
DTYPE_F16 = 1
DTYPE_F32 = 2

HADAMARD = 1
SMOOTH_K = 2
V_MMA_ORDER = 4
EXPCAST = 1
EXPCAST_EXACT = 2


class NativeUnavailable(RuntimeError):
    """libvcattn.so could not be loaded."""


class VCAttnError(RuntimeError):
    """A libvcattn entry point returned a non-zero status."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed with status {code}: {msg}")
        self.fn = fn
        self.code = code


class BHND(Structure):
    """vcattn_bhnd: a strided (B, H, N, D) view, strides in elements."""
    _fields_ = [("data", c_void_p), ("sb", c_int64), ("sh", c_int64), ("sn", c_int64)]


class RouteStats(Structure):
    """vcattn_route_stats."""
    _fields_ = [("q_block", c_int), ("k_mean", c_void_p), ("q_cent", c_void_p),
                ("q_bar", c_void_p), ("v_mean", c_void_p), ("sm_scale", c_float)]


_SIGNATURES = {
    "vcattn_abi_version": (c_int, []),
    "vcattn_last_error": (c_char_p, []),
    "vcattn_inject_fault": (None, [c_char_p]),
    "vcattn_inject_stall": (None, [c_int]),
    "vcattn_kmeans_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int]),
    "vcattn_kmeans": (c_int, [POINTER(BHND), c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                              c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p,
                              c_void_p, c_size_t, c_void_p]),
    "vcattn_prepare_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "vcattn_prepare_fp8": (c_int, [POINTER(BHND), POINTER(BHND), POINTER(BHND), c_int, c_int, c_int,
                                   c_int, c_int, c_void_p, c_int, c_int, c_int,
                                   c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                   c_void_p, c_void_p, POINTER(RouteStats), c_void_p, c_size_t,
                                   c_void_p]),
    "vcattn_attn_nvfp4": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                  c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_float,
                                  c_int, c_double, c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p]),
    "vcattn_prepare_nvfp4": (c_int, [POINTER(BHND), POINTER(BHND), c_int, c_int, c_int, c_int, c_int,
                                     c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                     c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                     c_size_t, c_void_p]),
    "vcattn_prepare_fp8_noalloc": (c_int, [POINTER(BHND), POINTER(BHND), POINTER(BHND), c_int, c_int,
                                           c_int, c_int, c_int, c_void_p, c_int, c_int, c_int,
                                           c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                           c_void_p, c_void_p, POINTER(RouteStats), c_void_p]),
    "vcattn_route_mask": (c_int, [POINTER(RouteStats), c_int, c_int, c_int, c_int, c_int, c_float,
                                  c_int, c_int, c_float, c_void_p, c_void_p, c_void_p]),
    "vcattn_attn_fp8": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                c_int, c_int, c_int, c_int, c_int, c_int, c_float, c_int, c_double,
                                c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p]),
    "vcattn_attn_split_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int, c_int, c_int]),
    "vcattn_attn_fp8_split": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                      c_int, c_int, c_int, c_int, c_int, c_int, c_float, c_int, c_double,
                                      c_void_p, c_int, c_int64, c_int64, c_int64, c_int, c_void_p, c_size_t,
                                      c_void_p]),
    "vcattn_attn_fp8_masked": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                       c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_float, c_int,
                                       c_double, c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p]),
    "vcattn_attn_fp8_mma": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                    c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_float,
                                    c_int, c_double, c_void_p, c_int, c_int64, c_int64, c_int64,
                                    c_void_p]),
    "vcattn_attn_status": (c_int, [POINTER(c_int), POINTER(c_int), POINTER(c_int), c_int]),
    "vcattn_attn_fp8_sparse": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                       c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                       c_int, c_int, c_int, c_int, c_int, c_int, c_float, c_int,
                                       c_double, c_void_p, c_int, c_int64, c_int64, c_int64,
                                       c_void_p]),
    "vcattn_route_tiles": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "vcattn_attn_fp8_sparse_tc": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                          c_void_p, c_void_p, c_void_p, c_int, c_int,
                                          c_int, c_int, c_int, c_int, c_int, c_int, c_float, c_int,
                                          c_double, c_void_p, c_int, c_int64, c_int64, c_int64,
                                          c_void_p]),
    "vcattn_e4m3_encode": (c_int, [c_void_p, c_int64, c_void_p, c_void_p]),
    "vcattn_fp4_encode": (c_int, [c_void_p, c_int64, c_void_p, c_void_p]),
    "vcattn_expcast_codes": (c_int, [c_void_p, c_void_p, c_int, c_int, c_double, c_int, c_void_p,
                                     c_void_p]),
}

_lock = threading.Lock()
_lib: Optional[ctypes.CDLL] = None
_load_error: Optional[str] = None


def lib() -> ctypes.CDLL:
    """The loaded library; raises NativeUnavailable (never falls back)."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            _load_error = (f"{LIB_PATH} not found; build it with "
                           f"`python -m comfyui_vc_attention_b200.build`")
            raise NativeUnavailable(_load_error)
        try:
            handle = ctypes.CDLL(LIB_PATH)
        except OSError as e:
            _load_error = f"failed to load {LIB_PATH}: {e}"
            raise NativeUnavailable(_load_error) from e
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
        return _lib


def available() -> bool:
    try:
        lib()
        return True
    except NativeUnavailable:
        return False


def load_error() -> Optional[str]:
    if _lib is None and _load_error is None:
        available()
    return _load_error


def check(fn: str, code: int) -> None:
    if code != OK:
        msg = lib().vcattn_last_error()
        raise VCAttnError(fn, code, msg.decode() if msg else "")


def inject_fault(entry_point: Optional[str]) -> None:
    """Host-side fault injection: make one entry point fail with ERR_INJECTED."""
    lib().vcattn_inject_fault(entry_point.encode() if entry_point else None)


def inject_stall(tile: int) -> None:
    """Bounded-wait test hook: the dense tcgen05 kernel issues no copies from
    KV tile ``tile`` on, so the waits on it give up (after about 2 s) and
    report through vcattn_attn_status; ``tile=-1`` clears it."""
    lib().vcattn_inject_stall(int(tile))


def declared_symbols(header: str = HEADER_PATH):
    """Function names declared in include/vcattn.h."""
    import re
    with open(header) as f:
        text = f.read()
    return sorted(set(re.findall(r"VCATTN_API\s+[\w\s\*]+?\b(vcattn_\w+)\s*\(", text)))
