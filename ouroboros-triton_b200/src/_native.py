"""ctypes binding of libouroboros_b200.so (declared in include/ouroboros_b200.h).

This module is the only place that touches the shared library. It never
falls back to anything: if the library is missing or a symbol is absent the
first call raises RuntimeError naming the build command.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "kernels" / "libouroboros_b200.so"

OURO_OK = 0
OURO_EINVAL = -1
OURO_EALLOC = -2
OURO_EUNSUPPORTED = -3
OURO_ECUDA = -4
OURO_EPAGETABLE = -5

DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2

_i32 = ctypes.c_int32
_pi32 = ctypes.POINTER(ctypes.c_int32)
_vp = ctypes.c_void_p

# name -> (restype, argtypes). Every symbol the header declares is listed, so
# a stale library fails at load time instead of mid-run.
_SIGNATURES: dict[str, tuple] = {
    "ouro_last_error": (ctypes.c_char_p, []),
    "ouro_version": (ctypes.c_char_p, []),
    "ouro_bt_create": (ctypes.c_int, [_i32, ctypes.POINTER(_vp)]),
    "ouro_bt_destroy": (None, [_vp]),
    "ouro_bt_max_blocks": (_i32, [_vp]),
    "ouro_bt_num_free": (_i32, [_vp]),
    "ouro_bt_is_allocated": (_i32, [_vp, _i32]),
    "ouro_bt_allocate_block": (ctypes.c_int, [_vp, _pi32]),
    "ouro_bt_free_block": (ctypes.c_int, [_vp, _i32]),
    "ouro_bt_link": (ctypes.c_int, [_vp, _i32, _i32]),
    "ouro_bt_allocate_chain": (ctypes.c_int, [_vp, _i32, _pi32]),
    "ouro_bt_expand_chain": (ctypes.c_int, [_vp, _i32, _pi32]),
    "ouro_bt_chain_len": (ctypes.c_int, [_vp, _i32, _pi32]),
    "ouro_bt_chain_tail": (ctypes.c_int, [_vp, _i32, _pi32]),
    "ouro_bt_walk": (ctypes.c_int, [_vp, _i32, _pi32, _i32, _pi32]),
    "ouro_bt_resolve_block": (ctypes.c_int, [_vp, _i32, _i32, _pi32]),
    "ouro_bt_free_chain": (ctypes.c_int, [_vp, _i32, _pi32]),
    "ouro_bt_export_page_table": (ctypes.c_int, [_vp, _pi32, _i32, _i32, _pi32]),
    "ouro_bt_next": (ctypes.c_int, [_vp, _i32, _pi32]),
    "ouro_bt_snapshot": (ctypes.c_int, [_vp, _pi32, ctypes.POINTER(ctypes.c_uint8), _pi32]),
    "ouro_bt_payload": (ctypes.c_int, [_vp, _i32, ctypes.POINTER(_pi32)]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def register(name: str, restype, argtypes) -> None:
    """Adds a symbol to the table checked at load time (used by kernel modules)."""
    _SIGNATURES[name] = (restype, argtypes)
    if _lib is not None:
        _bind(_lib, name)


def _bind(lib: ctypes.CDLL, name: str) -> None:
    try:
        fn = getattr(lib, name)
    except AttributeError as exc:
        raise RuntimeError(
            f"{LIB_PATH.name} does not export {name}; rebuild with "
            "`python ouroboros-triton_b200/build.py`"
        ) from exc
    restype, argtypes = _SIGNATURES[name]
    fn.restype = restype
    fn.argtypes = argtypes


def lib() -> ctypes.CDLL:
    """The loaded library (loaded once per process)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"native library {LIB_PATH} is not built; run "
                    "`python ouroboros-triton_b200/build.py` (needs nvcc)"
                )
            handle = ctypes.CDLL(str(LIB_PATH))
            for name in _SIGNATURES:
                _bind(handle, name)
            _lib = handle
    return _lib


def last_error() -> str:
    msg = lib().ouro_last_error()
    return msg.decode("utf-8", "replace") if msg else ""


def check(status: int, what: str = "") -> None:
    """Raises RuntimeError carrying the library's message for a non-zero status."""
    if status != OURO_OK:
        msg = last_error() or f"{what} failed with status {status}"
        raise RuntimeError(msg)


def exported_symbols() -> list[str]:
    return sorted(_SIGNATURES)
