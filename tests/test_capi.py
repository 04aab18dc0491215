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


def _attention_args(**over):
    """A filled ouro_attention_args with placeholder (never dereferenced) device addresses."""
    from src.kernels import _capi

    a = _capi.AttentionArgs()
    base = 1 << 32
    for i, f in enumerate(("q", "k_cache", "v_cache", "page_table", "seq_lens", "q_start", "cos",
                           "sin", "out")):
        setattr(a, f, base + i * (1 << 20))
    a.num_seqs, a.num_q_heads, a.num_kv_heads, a.head_dim, a.q_len = 2, 32, 8, 128, 256
    a.max_blocks, a.num_phys_blocks, a.max_positions = 16, 64, 1024
    a.dtype, a.causal, a.kernel = _native.DTYPE_BF16, 1, 0
    for k, v in over.items():
        setattr(a, k, v)
    return a


def _plan(a):
    lib = _native.lib()
    need, tc = ctypes.c_size_t(), ctypes.c_int32()
    rc = lib.ouro_attention_plan(ctypes.byref(a), ctypes.byref(need), ctypes.byref(tc))
    return rc, need.value, tc.value


def test_attention_plan_checks_arguments_on_the_host():
    assert _plan(_attention_args())[0] == _native.OURO_OK
    rc, _, _ = _plan(_attention_args(scope_tags=1 << 33, scope_stride=1024))
    assert rc == _native.OURO_EINVAL and "scope_lo" in _native.last_error()
    rc, _, _ = _plan(_attention_args(scope_tags=1 << 33, scope_stride=1000, scope_lo=1 << 34,
                                     scope_hi=1 << 35))
    assert rc == _native.OURO_EINVAL and "multiple of 16" in _native.last_error()
    rc, _, _ = _plan(_attention_args(scope_tags=(1 << 33) + 4, scope_stride=1024,
                                     scope_lo=1 << 34, scope_hi=1 << 35))
    assert rc == _native.OURO_EINVAL and "aligned" in _native.last_error()
    rc, _, _ = _plan(_attention_args(scope_tags=1 << 33, scope_stride=1024, scope_lo=1 << 34,
                                     scope_hi=1 << 35))
    assert rc == _native.OURO_OK
