"""The C-ABI library loads on a CPU-only host and exports every declared symbol."""

import ctypes
import re
from pathlib import Path

from src import _native
from src.kernels import block_attention  # noqa: F401  (registers the kernel symbols)

HEADERS = sorted((Path(__file__).resolve().parents[1] / "include").glob("*.h"))


def _declared():
    names = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(ouro_[a-z0-9_]+)\s*\(", text))
    return names


def test_every_declared_symbol_is_exported():
    lib = ctypes.CDLL(str(_native.LIB_PATH))
    declared = _declared()
    assert len(declared) > 20
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_header():
    assert _declared() <= set(_native.exported_symbols())


def test_version_and_error_plumbing():
    lib = _native.lib()
    assert b"sm_100a" in lib.ouro_version()
    h = ctypes.c_void_p()
    assert lib.ouro_bt_create(0, ctypes.byref(h)) == _native.OURO_EALLOC
    assert "max_blocks" in _native.last_error()
