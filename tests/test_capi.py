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


def _cpu_decode_inputs(S=4, hq=64, hkv=8, d=128, max_b=512, n_phys=4096):
    import torch

    return dict(page_table=torch.zeros((S, max_b), dtype=torch.int32),
                q=torch.zeros((S, hq, d), dtype=torch.bfloat16),
                k_cache=torch.zeros((8, hkv, 64, d), dtype=torch.bfloat16),
                v_cache=torch.zeros((8, hkv, 64, d), dtype=torch.bfloat16),
                seq_lens=torch.zeros(S, dtype=torch.int32),
                cos=torch.zeros((max_b * 64, d // 2)), sin=torch.zeros((max_b * 64, d // 2)),
                n_phys=n_phys)


def _decode_plan_of(S, total_blocks=0, max_seq_blocks=0, split=0, kernel="auto"):
    """The Python argument builder, then the library's planner (no device access)."""
    from src.kernels import block_attention as ba

    x = _cpu_decode_inputs(S=S)
    a = ba._decode_args(x["page_table"], x["q"], x["k_cache"], x["v_cache"], x["seq_lens"],
                        x["cos"], x["sin"], None, None, None, False, None, split, kernel,
                        torch_empty_like(x["q"]), None, None, total_blocks, max_seq_blocks)
    a.num_phys_blocks = x["n_phys"]
    return ba.decode_plan(a)


def torch_empty_like(t):
    import torch

    return torch.empty_like(t)


def test_decode_planner_sizes_chunks_from_the_real_work():
    """The split-K planner on the workload shape (GQA 64/8, D 128, 512-block rows):
    with total_blocks it plans from the batch's blocks, and max_seq_blocks bounds the
    chunks per sequence (so the workspace) instead of the page-table width."""
    wide = _decode_plan_of(256)
    real = _decode_plan_of(256, total_blocks=256 * 320, max_seq_blocks=512)
    small = _decode_plan_of(32, total_blocks=32 * 320, max_seq_blocks=512)
    assert real["split_blocks"] < wide["split_blocks"]
    assert small["split_blocks"] < real["split_blocks"]
    bounded = _decode_plan_of(32, total_blocks=32 * 320, max_seq_blocks=200)
    assert bounded["max_splits"] == -(-200 // bounded["split_blocks"])
    assert bounded["workspace_bytes"] < small["workspace_bytes"]


def test_decode_plan_rejects_negative_hints():
    from src import _native as nat

    try:
        _decode_plan_of(4, total_blocks=-1)
    except RuntimeError as exc:
        assert "total_blocks" in str(exc)
    else:
        raise AssertionError("negative total_blocks accepted")
    assert nat.last_error()


def test_rows_argument_builder_marshals_every_field():
    """The Python builder of ouro_attention_args runs end to end (paged queries with a
    bias and a block mask, and a dense chunk), and the library plans both."""
    import torch

    from src.kernels import block_attention as ba

    S, H, D, max_b = 2, 2, 128, 3
    q = torch.zeros((16, H, 64, D), dtype=torch.float16)
    pt = torch.zeros((S, max_b), dtype=torch.int32)
    lens = torch.tensor([192, 150], dtype=torch.int32)
    cos = torch.zeros((max_b * 64, D // 2))
    bias = torch.zeros((1, H, 192, 192))
    mask = torch.ones((S, 3, 3), dtype=torch.int8)
    out = torch.zeros((S, H, 192, D), dtype=torch.float16)
    a = ba._rows_args(q, True, q, q, pt, lens, None, cos, cos, (bias, (0, 192 * 192, 192, 1)),
                      (mask, (9, 3, 1)), out, None, H, 192, False, None, "auto")
    lib = _native.lib()
    need, tc = ctypes.c_size_t(), ctypes.c_int32()
    assert lib.ouro_attention_plan(ctypes.byref(a), ctypes.byref(need), ctypes.byref(tc)) == 0
    assert tc.value == 0   # an additive bias runs on the CUDA cores
    dense = ba._rows_args(torch.zeros((S, H, 128, D), dtype=torch.bfloat16), False,
                          q.bfloat16(), q.bfloat16(), pt, lens, torch.zeros(S, dtype=torch.int32),
                          cos, cos, None, None, torch.zeros((S, H, 128, D), dtype=torch.bfloat16),
                          None, H, 128, True, None, "auto")
    assert lib.ouro_attention_plan(ctypes.byref(dense), ctypes.byref(need),
                                   ctypes.byref(tc)) == 0


def test_scope_tags_in_kernel_layout_are_used_in_place():
    """Decode's token scope: uint8 tags whose rows are a multiple of 16 bytes, contiguous
    and 16-byte aligned are handed to the kernel as they are (the serving engine's per-slot
    tags); anything else is copied into a zero-padded [S, 16 k] buffer."""
    import torch

    from src.kernels.block_attention import _scope_tensors

    dev = torch.device("cpu")
    tags = torch.zeros(4, 32, dtype=torch.uint8)
    span = torch.zeros(4, 2, dtype=torch.int32)
    t, s = _scope_tensors((tags, span), 4, dev)
    assert t.data_ptr() == tags.data_ptr() and s.data_ptr() == span.data_ptr()
    ragged = torch.ones(4, 20, dtype=torch.bool)
    t2, _ = _scope_tensors((ragged, span), 4, dev)
    assert tuple(t2.shape) == (4, 32) and t2.dtype == torch.uint8
    assert t2[:, :20].all() and not t2[:, 20:].any()
    t3, _ = _scope_tensors((tags[:, :16], span), 4, dev)   # rows not contiguous: copied
    assert t3.data_ptr() != tags.data_ptr() and tuple(t3.shape) == (4, 16)
