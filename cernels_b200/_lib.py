"""ctypes binding of the C ABI in ``include/cernels_b200.h``.

The shared library is built in-tree (``cernels_b200/_C/libcernels_b200.so``) by
``cernels_b200.build``. There is no fallback: when the library is missing or cannot be
loaded every operator raises, so a run can never silently measure something else.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "_C" / "libcernels_b200.so"
_lock = threading.Lock()
_lib = None

LAYOUT_LINEAR = 0
LAYOUT_GPTOSS = 1

# Exported symbols and their prototypes (restype, argtypes), matching include/cernels_b200.h.
_VP = ctypes.c_void_p
_I32 = ctypes.c_int32
_SZ = ctypes.c_size_t


class MoeShape(ctypes.Structure):
    _fields_ = [
        ("tokens", ctypes.c_int32),
        ("hidden", ctypes.c_int32),
        ("experts", ctypes.c_int32),
        ("intermediate", ctypes.c_int32),
        ("topk", ctypes.c_int32),
        ("layout", ctypes.c_int32),
    ]


_SHAPE_P = ctypes.POINTER(MoeShape)

PROTOTYPES = {
    "cernels_error_string": (ctypes.c_char_p, [ctypes.c_int]),
    "cernels_version": (ctypes.c_int, []),
    "cernels_set_wait_limit_ns": (ctypes.c_int, [ctypes.c_uint64]),
    "cernels_moe_workspace_bytes": (ctypes.c_int, [_SHAPE_P, ctypes.c_int, ctypes.POINTER(_SZ)]),
    "cernels_moe_experts": (ctypes.c_int, [_SHAPE_P, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _SZ, _VP]),
    "cernels_moe_experts_decode": (ctypes.c_int, [_SHAPE_P, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _SZ, _VP]),
    "cernels_moe_experts_profiled": (ctypes.c_int, [_SHAPE_P, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _SZ, _VP,
                                                     ctypes.POINTER(ctypes.c_float)]),
    "cernels_moe_experts_decode_noalloc": (ctypes.c_int, [_SHAPE_P, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP]),
    "cernels_moe_grouped_experts": (ctypes.c_int, [_SHAPE_P, _I32, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _SZ, _VP]),
    "cernels_router": (ctypes.c_int, [_VP, _I32, _I32, _VP, _I32, _VP, _I32, _I32, _I32, _I32, _I32, _VP, _VP, _VP,
                                      _VP]),
    "cernels_router_topk": (ctypes.c_int, [_VP, _I32, _I32, _I32, _I32, _I32, _I32, _I32, _VP, _VP, _VP]),
    "cernels_moe_experts_shared": (ctypes.c_int, [_SHAPE_P, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _SZ, _VP]),
    "cernels_ep_create": (ctypes.c_int, [_I32, _I32, _I32, _I32, _I32, _I32, ctypes.POINTER(_VP), _VP]),
    "cernels_ep_connect": (ctypes.c_int, [_VP, ctypes.c_char_p]),
    "cernels_ep_destroy": (ctypes.c_int, [_VP]),
    "cernels_ep_dispatch": (ctypes.c_int, [_VP, _VP, _VP, _VP, _I32, _I32, ctypes.c_uint32, _VP]),
    "cernels_ep_experts_workspace_bytes": (ctypes.c_int, [_VP, _SHAPE_P, ctypes.POINTER(_SZ)]),
    "cernels_ep_experts": (ctypes.c_int, [_VP, _SHAPE_P, _VP, _VP, _VP, _VP, _VP, _VP, _I32, ctypes.c_uint32, _VP,
                                          _SZ, _VP]),
    "cernels_ep_combine": (ctypes.c_int, [_VP, _VP, _VP, _I32, _I32, _I32, _VP, ctypes.c_uint32, _VP]),
    "cernels_ep_status": (ctypes.c_int, [_VP, ctypes.POINTER(ctypes.c_int)]),
    "cernels_moe_route": (ctypes.c_int, [_SHAPE_P, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _SZ, _VP]),
    "cernels_moe_gather": (ctypes.c_int, [_VP, _VP, _I32, _I32, _VP, _VP]),
    "cernels_moe_combine": (ctypes.c_int, [_VP, _VP, _VP, _I32, _I32, _I32, _VP, _VP]),
    "cernels_workspace_status": (ctypes.c_int, [_SHAPE_P, ctypes.c_int, _VP, ctypes.POINTER(ctypes.c_int), _VP]),
}


class CernelsError(RuntimeError):
    """Raised when a C-ABI call returns a nonzero code (the reference raises c10::Error)."""


def lib_path() -> Path:
    return Path(os.environ.get("CERNELS_B200_LIB", str(_LIB_PATH)))


def load():
    """Loads (once) and returns the ctypes library with prototypes applied."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = lib_path()
        if not path.exists():
            raise CernelsError(
                f"cernels_b200 native library not found at {path}; build it with "
                "`python -m cernels_b200.build` (there is no CPU or eager fallback)"
            )
        lib = ctypes.CDLL(str(path))
        for name, (res, args) in PROTOTYPES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def check(code: int, what: str) -> None:
    if code != 0:
        msg = load().cernels_error_string(code).decode()
        raise CernelsError(f"{what} failed: {msg} (code {code})")


def workspace_bytes(shape: MoeShape, decode: bool) -> int:
    n = _SZ(0)
    check(load().cernels_moe_workspace_bytes(ctypes.byref(shape), int(decode), ctypes.byref(n)), "workspace query")
    return int(n.value)
