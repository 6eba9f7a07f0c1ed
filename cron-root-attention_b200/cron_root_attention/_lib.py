"""ctypes binding of libcra.so, the C ABI declared in include/cra.h.

The library is built in-tree (``cron-root-attention_b200/build.py``) next to
this file.  There is no fallback: if the library is missing or fails to load,
every call raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libcra.so")

CRA_F16 = 0
CRA_BF16 = 1

_lock = threading.Lock()
_lib = None

_i64p = ctypes.POINTER(ctypes.c_int64)
_vp = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float

_SIGNATURES = {
    "cra_status_string": (ctypes.c_char_p, [_i]),
    "cra_version": (_i, []),
    "cra_last_error_message": (ctypes.c_char_p, []),
    "cra_window": (_i, [ctypes.c_int64]),
    "cra_relay_active": (_i, [ctypes.c_int64]),
    "cra_global_rows": (ctypes.c_int64, [ctypes.c_int64, _i, _i]),
    "cra_relay_build": (_i, [_vp, _vp, _i64p, _i64p, _i, _i, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp]),
    "cra_fwd": (_i, [_vp, _vp, _vp, _vp, _vp, _i64p, _i64p, _i64p, _i, _i, _i, _i, _i, _i, _i, _i, _f, _vp,
                     _i64p, _vp, _vp, _vp]),
    "cra_relay_build_shard": (_i, [_vp, _vp, _i64p, _i64p, _i, _i, ctypes.c_int64, ctypes.c_int64, _i, _i, _i, _i, _i,
                                   _vp, _vp, _vp, _vp, _vp]),
    "cra_fwd_shard": (_i, [_vp, _vp, _vp, _vp, _vp, _i64p, _i64p, _i64p, _i, _i, _i, ctypes.c_int64, ctypes.c_int64,
                           _i, ctypes.c_int64, _i, _vp, _vp, _i64p, _i64p, ctypes.c_int64, _i,
                           _i, _i, _i, _i, _f, _vp, _i64p, _vp, _vp, _vp]),
    "cra_varlen_table_bytes": (ctypes.c_size_t, [_i]),
    "cra_varlen_global_rows": (ctypes.c_int64, [_i64p, _i, _i]),
    "cra_varlen_blocks": (ctypes.c_int64, [_i64p, _i]),
    "cra_varlen_plan": (_i, [_i64p, _i, _i, _vp, _vp]),
    "cra_relay_build_varlen": (_i, [_vp, _vp, _i64p, _i64p, _i, _i, _i64p, _i, _vp, _i, _i, _i, _vp, _vp, _vp, _vp,
                                    _vp]),
    "cra_fwd_varlen": (_i, [_vp, _vp, _vp, _vp, _vp, _i64p, _i64p, _i64p, _i, _i, _i, _i64p, _i, _vp, _i, _i, _i, _f,
                            _vp, _i64p, _vp, _vp, _vp]),
    "cra_bwd_shard_workspace_bytes": (ctypes.c_size_t, [_i, _i, _i, ctypes.c_int64, _i, _i, _i, _i]),
    "cra_bwd_shard_global": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i64p, _i64p, _i64p, _i, _i, _i, ctypes.c_int64,
                                  ctypes.c_int64, _i, _i, _i, _i, _i, _f, _vp, _vp, _vp, ctypes.c_size_t, _vp, _vp]),
    "cra_bwd_shard_local": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64p, _i64p, _i64p, _i64p, _vp, _vp, _i64p, _i64p,
                                 ctypes.c_int64, _i, _i, _i, _i, ctypes.c_int64, ctypes.c_int64, _i, _i, _i, _i, _i,
                                 _f, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64p, _i64p, _i64p, _i64p, _i64p, _vp,
                                 _vp, ctypes.c_size_t, _vp, _vp]),
    "cra_bwd_workspace_bytes": (ctypes.c_size_t, [_i, _i, _i, _i, _i, _i, _i]),
    "cra_bwd_fused_workspace_bytes": (ctypes.c_size_t, [_i, _i, _i, _i, _i, _i, _i]),
    "cra_bwd": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64p, _i64p, _i64p, _i64p, _i64p,
                     _i, _i, _i, _i, _i, _i, _i, _i, _f, _vp, _vp, _vp, _vp, _i64p, _i64p, _i64p, _vp, _vp,
                     ctypes.c_size_t, _vp, _vp]),
    "cra_bwd_kernel_times": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64p, _i64p, _i64p, _i64p, _i64p,
                                  _i, _i, _i, _i, _i, _i, _i, _i, _f, _vp, _vp, _vp, _vp, _i64p, _i64p, _i64p, _vp,
                                  _vp, ctypes.c_size_t, _vp, _vp, ctypes.POINTER(_f),
                                  ctypes.POINTER(ctypes.c_char_p), _i, ctypes.POINTER(_i), _i]),
    "cra_bwd_fused": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64p, _i64p, _i64p, _i64p, _i64p,
                                   _i, _i, _i, _i, _i, _i, _i, _i, _f, _vp, _vp, _vp, _vp, _i64p, _i64p, _i64p,
                                   _vp, _vp, ctypes.c_size_t, _vp, _vp]),
    "cra_bwd_noalloc": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64p, _i64p, _i64p, _i64p, _i64p,
                             _i, _i, _i, _i, _i, _i, _i, _i, _f, _vp, _vp, _vp, _vp, _i64p, _i64p, _i64p, _vp,
                             _vp, _vp]),
}

# Every symbol include/cra.h declares (checked by the CPU test suite).
EXPORTED = tuple(_SIGNATURES)


class CraError(RuntimeError):
    """A non-zero status returned by libcra."""


def lib():
    """Load libcra.so once and return the ctypes handle (raises if absent)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"libcra.so not found at {LIB_PATH}; build it with "
                        "`python cron-root-attention_b200/build.py` (no CPU fallback exists)")
                h = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in _SIGNATURES.items():
                    fn = getattr(h, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = h
    return _lib


def check(status: int, what: str) -> None:
    if status != 0:
        msg = lib().cra_status_string(status).decode()
        detail = lib().cra_last_error_message().decode()
        raise CraError(f"{what} failed: {msg} (status {status}): {detail}")


def strides3(t) -> ctypes.Array:
    """(batch, head, seq) element strides of a [B, H, S, D] tensor."""
    s = t.stride()
    return (ctypes.c_int64 * 3)(s[0], s[1], s[2])
