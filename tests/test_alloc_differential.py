"""Lockstep differential: native allocator vs the reference's recorded results.

The op scripts in tests/golden/alloc_scripts.json were run through the
reference's Python BlockTable by make_golden.py (links are only taken when
they keep chains acyclic, so every script terminates). Each op is replayed
here against (a) the native allocator behind src.block_table, (b) the plain
Python restatement in oracle/, and (c) the reference's own C++ allocator
compiled into oracle/_ref when it is present; results, error texts and the
final state must match exactly.
"""

import ctypes
import json
from pathlib import Path

import pytest

from oracle.block_table_oracle import OracleBlockTable
from src.block_table import BlockTable

GOLDEN = Path(__file__).resolve().parent / "golden" / "alloc_scripts.json"
REF_LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libref_block_table.so"
SCRIPTS = json.loads(GOLDEN.read_text())


def _apply(bt, op):
    kind = op[0]
    if kind == "alloc":
        return bt.allocate_block()
    if kind == "free":
        return bt.free_block(op[1])
    if kind == "chain":
        return bt.allocate_chain(op[1])
    if kind == "expand":
        return bt.expand_chain(op[1])
    if kind == "link":
        return bt.link(op[1], op[2])
    if kind == "walk":
        return list(bt.walk(op[1]))
    if kind == "len":
        return bt.chain_len(op[1])
    if kind == "resolve":
        return bt.resolve_block(op[1], op[2])
    if kind == "row":
        return list(bt.page_table_row(op[1], pad_to=op[2]))
    if kind == "cell":
        bt.set_cell(op[1], op[2], op[3])
        return bt.get_cell(op[1], op[2])
    raise AssertionError(kind)


class _RefCpp:
    """The reference's C++ BlockTable through oracle/ref_block_table_shim.cpp."""

    def __init__(self, lib, n):
        self.lib, self.h = lib, ctypes.c_void_p(lib.ref_create(n))
        self.n = n

    def _call(self, fn, *args, out=True):
        o = ctypes.c_int()
        rc = fn(self.h, *args, ctypes.byref(o)) if out else fn(self.h, *args)
        if rc != 0:
            raise RuntimeError(self.lib.ref_last_error().decode())
        return o.value if out else None

    def allocate_block(self):
        return self._call(self.lib.ref_allocate_block)

    def free_block(self, i):
        return self._call(self.lib.ref_free_block, i, out=False)

    def allocate_chain(self, n):
        return self._call(self.lib.ref_allocate_chain, n)

    def expand_chain(self, t):
        return self._call(self.lib.ref_expand_chain, t)

    def link(self, a, b):
        return self._call(self.lib.ref_link, a, b, out=False)

    def chain_len(self, h):
        return self._call(self.lib.ref_chain_len, h)

    def resolve_block(self, h, i):
        return self._call(self.lib.ref_resolve_block, h, i)

    def set_cell(self, i, off, v):
        return self._call(self.lib.ref_set_cell, i, off, v, out=False)

    def get_cell(self, i, off):
        return self._call(self.lib.ref_get_cell, i, off)

    def _list(self, fn, *args):
        buf, n = (ctypes.c_int * (self.n + 64))(), ctypes.c_int()
        if fn(self.h, *args, buf, self.n + 64, ctypes.byref(n)) != 0:
            raise RuntimeError(self.lib.ref_last_error().decode())
        return list(buf[: n.value])

    def walk(self, h):
        return self._list(self.lib.ref_walk, h)

    def page_table_row(self, h, pad_to=None):
        return self._list(self.lib.ref_page_table_row, h, -1 if pad_to is None else pad_to)

    @property
    def num_free(self):
        return self.lib.ref_num_free(self.h)


def _ref_lib():
    if not REF_LIB.exists():
        return None
    lib = ctypes.CDLL(str(REF_LIB))
    lib.ref_create.restype = ctypes.c_void_p
    lib.ref_last_error.restype = ctypes.c_char_p
    for name in ("ref_allocate_block", "ref_free_block", "ref_link", "ref_allocate_chain",
                 "ref_expand_chain", "ref_chain_len", "ref_resolve_block", "ref_set_cell",
                 "ref_get_cell", "ref_walk", "ref_page_table_row", "ref_num_free"):
        getattr(lib, name).argtypes = None
    return lib


def _check_script(script, bt, *, exact_messages=True):
    for step in script["steps"]:
        op = step["op"]
        if step.get("skip"):
            continue
        try:
            got, err = _apply(bt, op), None
        except RuntimeError as exc:
            got, err = None, str(exc)
        if "error" in step:
            assert err is not None, f"{op}: expected error {step['error']!r}, got {got!r}"
            if exact_messages:
                assert err == step["error"], op
        else:
            assert err is None, f"{op}: unexpected error {err!r}"
            assert got == step["result"], op


@pytest.mark.parametrize("script", SCRIPTS, ids=[f"seed{s['seed']}" for s in SCRIPTS])
def test_native_allocator_matches_reference_script(script):
    bt = BlockTable(max_blocks=script["max_blocks"])
    _check_script(script, bt)
    fin = script["final"]
    assert bt.num_free == fin["num_free"]
    assert bt.next_ptr == fin["next_ptr"]
    assert bt.blocks == fin["payload"]
    assert bt.free_list == fin["free_list"]


@pytest.mark.parametrize("script", SCRIPTS, ids=[f"seed{s['seed']}" for s in SCRIPTS])
def test_oracle_restatement_matches_reference_script(script):
    bt = OracleBlockTable(script["max_blocks"])
    _check_script(script, bt)
    assert bt.state() == (script["final"]["num_free"], script["final"]["next_ptr"],
                          script["final"]["payload"], script["final"]["free_list"])


@pytest.mark.parametrize("script", SCRIPTS, ids=[f"seed{s['seed']}" for s in SCRIPTS])
def test_reference_cpp_allocator_matches_reference_script(script):
    lib = _ref_lib()
    if lib is None:
        pytest.skip("oracle/_ref not built (make -C oracle where the reference is mounted)")
    bt = _RefCpp(lib, script["max_blocks"])
    # The reference C++ words a few errors differently from its Python twin
    # (e.g. resolve_block omits "starting at head"); compare outcomes, not texts.
    _check_script(script, bt, exact_messages=False)
    assert bt.num_free == script["final"]["num_free"]


def test_large_pool_allocation_order_matches_oracle():
    import random
    rng = random.Random(5)
    n = 4096
    a, b = BlockTable(n), OracleBlockTable(n)
    ids = [a.allocate_block() for _ in range(n)]
    assert ids == [b.allocate_block() for _ in range(n)]
    rng.shuffle(ids)
    for i in ids:
        a.free_block(i)
        b.free_block(i)
    for k in (7, 130, 1, 64, 513):
        assert list(a.walk(a.allocate_chain(k))) == b.walk(b.allocate_chain(k))
    assert a.free_list == b.free_list
