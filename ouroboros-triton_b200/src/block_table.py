"""KV-block memory: 64-token physical blocks, chains and page tables.

Drop-in for the reference module ``src/block_table.py``: the same constants,
the same ``BlockTable`` methods and attributes, the same ``resolve_block`` and
``build_page_table`` helpers, the same error texts. The table itself lives in
native code (``csrc/block_table.cpp`` through the C ABI in
``include/ouroboros_b200.h``); this class is a thin handle over it, so the
Supervisor, the page-table export and the kernels all see one allocator.

Semantics kept from the reference (file:line of ``src/block_table.py``):
  * block id == slot index forever; a fresh table hands out 0, 1, 2, ... (:59-74)
  * ``allocate_chain`` is all-or-nothing (:112-130)
  * ``free_block`` zeroes the payload and rejects double frees (:89-94)
  * ``walk`` validates ``head`` at call time (:132-145)
  * ``page_table_row`` / ``build_page_table`` pad with ``PAD_ID`` (:187-222)

Differences, all additive:
  * ``walk`` returns the ids of the chain as it is at call time; a cycle made
    with ``link`` raises instead of looping forever;
  * ``export_page_table`` fills one contiguous int32 array for the device copy;
  * ``free_chain`` / ``chain_tail`` are single native calls.
"""

from __future__ import annotations

import ctypes
from typing import Iterable, Iterator, Sequence

import numpy as np

from . import _native

BLOCK_SIZE = 64  # tokens per physical block (reference block_table.py:13)
PAD_ID = -1  # page-table slot with no physical block (reference block_table.py:14)

_I32_MIN, _I32_MAX = -(2**31), 2**31 - 1

__all__ = [
    "BLOCK_SIZE",
    "PAD_ID",
    "BlockTable",
    "BlockPayload",
    "resolve_block",
    "build_page_table",
    "build_page_table_array",
]


def resolve_block(table, logical_idx: int) -> int:
    """Physical id at ``logical_idx`` of a 1-D page-table row.

    Same checks and messages as the reference free function
    (src/block_table.py:17-56).
    """
    if isinstance(table, BlockTable):
        raise RuntimeError(
            "resolve_block expects a 1-D page-table row; use "
            "BlockTable.resolve_block(head, logical_idx) for chain lookup"
        )
    try:
        n_slots = len(table)
    except TypeError:
        raise RuntimeError(
            f"page table row must be a finite sequence, got {type(table).__name__}"
        ) from None
    if isinstance(logical_idx, bool) or not isinstance(logical_idx, int):
        raise RuntimeError(f"invalid logical index: {logical_idx!r}")
    if logical_idx < 0 or logical_idx >= n_slots:
        raise RuntimeError(
            f"logical block {logical_idx} out of range for page table of {n_slots} slots"
        )
    phys = table[logical_idx]
    if phys == PAD_ID:
        raise RuntimeError(f"logical block {logical_idx} is padded (no physical block)")
    return int(phys) if isinstance(phys, (int, np.integer)) else phys


class BlockPayload:
    """Live view of one block's 64 payload cells (writes go to the table).

    Compares equal to any sequence with the same values, so
    ``bt.get_block(i) == [0] * 64`` reads as in the reference.
    """

    __slots__ = ("_owner", "_arr")

    def __init__(self, owner: "BlockTable", arr: np.ndarray):
        self._owner = owner
        self._arr = arr

    def __len__(self) -> int:
        return BLOCK_SIZE

    def __getitem__(self, i):
        v = self._arr[i]
        return v.tolist() if isinstance(v, np.ndarray) else int(v)

    def __setitem__(self, i, value) -> None:
        self._arr[i] = value

    def __iter__(self) -> Iterator[int]:
        return iter(self._arr.tolist())

    def __eq__(self, other) -> bool:
        try:
            return list(self) == list(other)
        except TypeError:
            return NotImplemented

    def __repr__(self) -> str:
        return f"BlockPayload({self._arr.tolist()!r})"

    def tolist(self) -> list[int]:
        return self._arr.tolist()


def _require_int(value, what: str) -> int:
    if isinstance(value, bool) or not isinstance(value, (int, np.integer)):
        raise RuntimeError(f"invalid {what}: {value!r}")
    return int(value)


class BlockTable:
    """Array-backed linked list of fixed 64-token blocks (native storage)."""

    def __init__(self, max_blocks: int = 1024):
        max_blocks = _require_int(max_blocks, "block count")
        if not (1 <= max_blocks <= _I32_MAX):
            raise RuntimeError("max_blocks must be >= 1")
        self._lib = _native.lib()
        handle = ctypes.c_void_p()
        _native.check(self._lib.ouro_bt_create(max_blocks, ctypes.byref(handle)), "create")
        self._h = handle
        self.max_blocks = max_blocks
        self.block_size = BLOCK_SIZE

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            self._lib.ouro_bt_destroy(h)
            self._h = None

    # -- helpers ---------------------------------------------------------
    def _id(self, idx) -> int:
        """Validates a block id argument; out-of-int32 ids are simply not allocated."""
        idx = _require_int(idx, "block id")
        if not (_I32_MIN <= idx <= _I32_MAX):
            raise RuntimeError(f"block {idx} is not allocated")
        return idx

    def _out(self, fn, *args) -> int:
        out = ctypes.c_int32()
        _native.check(fn(self._h, *args, ctypes.byref(out)))
        return out.value

    # -- single blocks -----------------------------------------------------
    def allocate_block(self) -> int:
        """Lowest-id-first LIFO allocation (reference block_table.py:76-87)."""
        return self._out(self._lib.ouro_bt_allocate_block)

    def free_block(self, idx: int) -> None:
        """Return a block to the free stack; double free raises (block_table.py:89-94)."""
        _native.check(self._lib.ouro_bt_free_block(self._h, self._id(idx)))

    def is_allocated(self, idx: int) -> bool:
        idx = self._id(idx)
        return bool(self._lib.ouro_bt_is_allocated(self._h, idx))

    def get_block(self, idx: int) -> BlockPayload:
        """Live payload view of an allocated block (block_table.py:96-99)."""
        idx = self._id(idx)
        ptr = ctypes.POINTER(ctypes.c_int32)()
        _native.check(self._lib.ouro_bt_payload(self._h, idx, ctypes.byref(ptr)))
        return BlockPayload(self, np.ctypeslib.as_array(ptr, shape=(BLOCK_SIZE,)))

    def set_cell(self, idx: int, offset: int, value: int) -> None:
        """Cell write, as in the C++ binding (bindings.cpp:36-47)."""
        self.get_block(idx)[_require_int(offset, "offset")] = value

    def get_cell(self, idx: int, offset: int) -> int:
        return self.get_block(idx)[_require_int(offset, "offset")]

    def link(self, prev_idx: int, next_idx: int) -> None:
        """next_ptr[prev] = next for two allocated blocks (block_table.py:101-105)."""
        _native.check(self._lib.ouro_bt_link(self._h, self._id(prev_idx), self._id(next_idx)))

    # -- chains ------------------------------------------------------------
    def allocate_chain(self, n_blocks: int) -> int:
        """All-or-nothing chain of ``n_blocks``; returns the head (block_table.py:112-130)."""
        if isinstance(n_blocks, bool) or not isinstance(n_blocks, (int, np.integer)):
            raise RuntimeError(f"invalid block count: {n_blocks!r}")
        n_blocks = int(n_blocks)
        if n_blocks <= 0:
            raise RuntimeError(f"chain length must be >= 1, got {n_blocks}")
        if n_blocks > _I32_MAX:
            raise RuntimeError(
                f"insufficient free blocks: requested {n_blocks}, {self.num_free} available"
            )
        return self._out(self._lib.ouro_bt_allocate_chain, n_blocks)

    def walk(self, head: int) -> Iterator[int]:
        """Block ids from ``head`` to the tail; ``head`` is validated now."""
        return iter(self._walk_list(self._id(head)))

    def _walk_list(self, head: int) -> list[int]:
        n = self.chain_len(head)
        buf = (ctypes.c_int32 * n)()
        got = ctypes.c_int32()
        _native.check(self._lib.ouro_bt_walk(self._h, head, buf, n, ctypes.byref(got)))
        return list(buf[: got.value])

    def chain_len(self, head: int) -> int:
        return self._out(self._lib.ouro_bt_chain_len, self._id(head))

    def chain_tail(self, head: int) -> int:
        return self._out(self._lib.ouro_bt_chain_tail, self._id(head))

    def expand_chain(self, tail: int) -> int:
        """[EXPAND]: one new block linked after ``tail`` (block_table.py:152-165)."""
        return self._out(self._lib.ouro_bt_expand_chain, self._id(tail))

    def free_chain(self, head: int) -> int:
        """Frees every block of the chain; returns how many were freed."""
        return self._out(self._lib.ouro_bt_free_chain, self._id(head))

    def resolve_block(self, head: int, logical_idx: int) -> int:
        """Physical id at ``logical_idx`` along the chain (block_table.py:167-185)."""
        head = self._id(head)
        n = self.chain_len(head)  # validates head first, as the reference does
        if isinstance(logical_idx, bool) or not isinstance(logical_idx, (int, np.integer)):
            raise RuntimeError(f"invalid logical index: {logical_idx!r}")
        logical_idx = int(logical_idx)
        if not (0 <= logical_idx < n):
            raise RuntimeError(
                f"logical block {logical_idx} out of range for chain of "
                f"{n} block(s) starting at head {head}"
            )
        return self._out(self._lib.ouro_bt_resolve_block, head, logical_idx)

    def page_table_row(self, head: int, pad_to: int | None = None) -> list[int]:
        """Chain ids, optionally right-padded with PAD_ID (block_table.py:187-199)."""
        head = self._id(head)
        if pad_to is None:
            return self._walk_list(head)
        return self.export_page_table([head], pad_to)[0].tolist()

    def export_page_table(self, heads: Sequence[int], pad_to: int,
                          out: np.ndarray | None = None) -> np.ndarray:
        """[len(heads), pad_to] int32 page table in one native call.

        ``out`` may be a preallocated C-contiguous int32 array (for example a
        numpy view of pinned host memory); it is returned filled.
        """
        ids = np.ascontiguousarray([self._id(h) for h in heads], dtype=np.int32)
        pad_to = _require_int(pad_to, "pad_to")
        if pad_to > _I32_MAX:
            raise RuntimeError("pad_to too large")
        pad_to = max(pad_to, _I32_MIN)
        n = int(ids.shape[0])
        if out is None:
            out = np.empty((n, max(pad_to, 0)), dtype=np.int32)
        elif (out.dtype != np.int32 or not out.flags["C_CONTIGUOUS"]
              or out.size < n * max(pad_to, 0)):
            raise RuntimeError("export_page_table: out must be a contiguous int32 buffer "
                               f"with room for {n}x{pad_to} entries")
        _native.check(self._lib.ouro_bt_export_page_table(
            self._h, ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), n, pad_to,
            out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))))
        return out

    # -- whole-table views ---------------------------------------------------
    def _snapshot(self):
        m = self.max_blocks
        nxt = np.empty(m, dtype=np.int32)
        live = np.empty(m, dtype=np.uint8)
        free = np.empty(self.num_free, dtype=np.int32)
        _native.check(self._lib.ouro_bt_snapshot(
            self._h, nxt.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
            live.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)),
            free.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))))
        return nxt, live, free

    @property
    def num_free(self) -> int:
        return int(self._lib.ouro_bt_num_free(self._h))

    @property
    def next_ptr(self) -> list[int]:
        """Snapshot of next_ptr per slot (-1 at tails and free slots)."""
        return self._snapshot()[0].tolist()

    @property
    def free_list(self) -> list[int]:
        """Snapshot of the LIFO free stack, bottom first (top is allocated next)."""
        return self._snapshot()[2].tolist()

    @property
    def blocks(self) -> list[list[int] | None]:
        """Snapshot: payload list per allocated slot, None for free slots."""
        _, live, _ = self._snapshot()
        return [self.get_block(i).tolist() if live[i] else None for i in range(self.max_blocks)]


def build_page_table(table: BlockTable, heads: Iterable[int],
                     pad_to: int | None = None) -> list[list[int]]:
    """One page-table row per chain head (reference block_table.py:212-222)."""
    return [table.page_table_row(h, pad_to=pad_to) for h in heads]


def build_page_table_array(table: BlockTable, heads: Iterable[int],
                           pad_to: int | None = None) -> np.ndarray:
    """Same rows as :func:`build_page_table` as one [S, pad_to] int32 array.

    ``pad_to`` defaults to the longest chain.
    """
    heads = list(heads)
    if pad_to is None:
        pad_to = max((table.chain_len(h) for h in heads), default=0)
    return table.export_page_table(heads, pad_to)
