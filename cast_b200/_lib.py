"""ctypes binding of ``libcast_b200.so`` (the C ABI in ``include/cast_b200.h``).

The library is loaded lazily on first use and never replaced by a Python or
CPU implementation: if it is missing, every operation raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libcast_b200.so")

_lock = threading.Lock()
_lib = None

c_int, c_float, c_size_t, c_void_p = ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_void_p
c_longlong = ctypes.c_longlong

# name -> (restype, argtypes); mirrors include/cast_b200.h
SIGNATURES = {
    "cast_status_string": (ctypes.c_char_p, [c_int]),
    "cast_last_error_message": (ctypes.c_char_p, []),
    "cast_version": (c_int, []),
    "cast_device_error": (c_int, [c_void_p]),
    "cast_selftest_bounded_wait": (c_int, [c_int, c_int, c_void_p]),
    "cast_rcsa_select_quant": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
         c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p, c_int, c_float, c_void_p, c_void_p, c_size_t, c_void_p],
    ),
    "cast_rcsa_select_quant_workspace_bytes": (c_size_t, [c_int] * 6),
    "cast_rcsa_select_quant_noalloc": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
         c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p, c_int, c_float, c_void_p, c_void_p],
    ),
    "cast_compact_select": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_int,
         c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_float,
         c_void_p, c_void_p, c_size_t, c_void_p],
    ),
    "cast_compact_select_workspace_bytes": (c_size_t, [c_int] * 5),
    "cast_taba_select": (
        c_int,
        [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
         c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p],
    ),
    "cast_taba_select_workspace_bytes": (c_size_t, [c_int] * 9),
    "cast_rcsa_attention": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
         c_float, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p],
    ),
    "cast_rcsa_attention_workspace_bytes": (c_size_t, [c_int] * 7 + [c_void_p]),
    "cast_rcsa_attention_peers": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
         c_float, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_int, c_void_p, c_void_p,
         c_void_p, c_void_p, c_void_p],
    ),
    "cast_peer_push": (c_int, [c_void_p, c_size_t, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "cast_peer_send": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p, c_void_p, c_void_p]),
    "cast_peer_alloc": (c_int, [c_size_t, c_void_p, c_void_p]),
    "cast_peer_open": (c_int, [c_void_p, c_void_p]),
    "cast_peer_close": (c_int, [c_void_p]),
    "cast_peer_free": (c_int, [c_void_p]),
    "cast_peer_wait": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "cast_compact_pack": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int,
         c_int, c_void_p, c_void_p, c_void_p, c_void_p],
    ),
    "cast_compact_unpack": (c_int, [c_void_p, c_void_p] + [c_int] * 5 + [c_void_p, c_void_p]),
    "cast_barycentric_pair_write": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_longlong, c_int,
         c_void_p],
    ),
    "cast_barycentric_weights": (
        c_int,
        [c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_int, c_int, c_void_p, c_int,
         c_int, c_void_p, c_int, c_int, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_float, c_float,
         c_void_p, c_void_p, c_void_p, c_void_p, c_void_p],
    ),
    "cast_swap_route": (
        c_int,
        [c_void_p] * 9 + [c_int] * 9 + [c_float, c_int, c_int, c_int, c_int, c_void_p, c_void_p,
                                         c_size_t, c_void_p],
    ),
    "cast_swap_objective": (
        c_int,
        [c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int,
         c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
         c_int, c_float, c_float, c_float, c_float, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p, c_void_p, c_void_p],
    ),
    "cast_swap_route_workspace_bytes": (c_size_t, [c_int] * 10),
    "cast_par_fcpasm": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_float,
         c_float, c_float, c_float, c_int, c_int, c_void_p, c_void_p, c_void_p, c_size_t,
         c_void_p],
    ),
    "cast_par_fcpasm_workspace_bytes": (c_size_t, [c_int] * 4),
}


class CastError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, status: int, name: str, message: str):
        super().__init__(f"{name}: {message}")
        self.status = status


def load():
    """Loads the library (once) and binds every declared symbol."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `python -m cast_b200.build` "
                    "(the hot path has no CPU fallback)"
                )
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(status: int, name: str) -> None:
    if status != 0:
        lib = load()
        msg = lib.cast_last_error_message().decode(errors="replace")
        kind = lib.cast_status_string(status).decode()
        raise CastError(status, name, f"{kind}: {msg}")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)


def check_device(stream: int | None, where: str) -> None:
    """Raises :class:`CastError` when a kernel reported a device-side error
    (a bounded wait that gave up, an index out of range) since the last
    check.  Synchronises ``stream``: call it where the caller synchronises
    anyway."""
    check(load().cast_device_error(stream), where)


def ptr(t) -> int | None:
    """Device pointer of a tensor (None for None)."""
    return None if t is None else t.data_ptr()
