"""CPU oracle for the KV-block allocator — TEST INFRASTRUCTURE ONLY.

A plain-Python restatement of the reference allocator
(src/block_table.py:59-209) used as the checker in lockstep differential
tests against the native allocator. Only tests may import it.

Each method cites the reference lines it restates. Walks here are bounded by
the pool size (a cycle raises) so a checker never hangs; the reference's
walk loops forever on a cycle (src/block_table.py:141-145).
"""

from __future__ import annotations

BLOCK_SIZE = 64
PAD_ID = -1


class OracleBlockTable:
    def __init__(self, max_blocks: int):
        # block_table.py:67-74 — slot arrays, reversed free stack
        self.max_blocks = max_blocks
        self.payload: list[list[int] | None] = [None] * max_blocks
        self.next_ptr: list[int] = [-1] * max_blocks
        self.free_list: list[int] = list(range(max_blocks - 1, -1, -1))

    def _require(self, idx: int) -> None:
        # block_table.py:201-205
        if idx < 0 or idx >= self.max_blocks or self.payload[idx] is None:
            raise RuntimeError(f"block {idx} is not allocated")

    @property
    def num_free(self) -> int:  # block_table.py:207-209
        return len(self.free_list)

    def allocate_block(self) -> int:  # block_table.py:76-87
        if not self.free_list:
            raise RuntimeError("No free blocks available")
        idx = self.free_list.pop()
        self.payload[idx] = [0] * BLOCK_SIZE
        self.next_ptr[idx] = -1
        return idx

    def free_block(self, idx: int) -> None:  # block_table.py:89-94
        self._require(idx)
        self.payload[idx] = None
        self.next_ptr[idx] = -1
        self.free_list.append(idx)

    def set_cell(self, idx: int, off: int, value: int) -> None:  # bindings.cpp:36-47
        self._require(idx)
        self.payload[idx][off] = value

    def get_cell(self, idx: int, off: int) -> int:
        self._require(idx)
        return self.payload[idx][off]

    def link(self, prev: int, nxt: int) -> None:  # block_table.py:101-105
        self._require(prev)
        self._require(nxt)
        self.next_ptr[prev] = nxt

    def allocate_chain(self, n: int) -> int:  # block_table.py:112-130
        if n <= 0:
            raise RuntimeError(f"chain length must be >= 1, got {n}")
        if len(self.free_list) < n:
            raise RuntimeError(
                f"insufficient free blocks: requested {n}, {len(self.free_list)} available")
        ids = [self.allocate_block() for _ in range(n)]
        for a, b in zip(ids, ids[1:]):
            self.next_ptr[a] = b
        return ids[0]

    def walk(self, head: int) -> list[int]:  # block_table.py:132-145
        self._require(head)
        out, idx = [], head
        while idx != -1:
            if len(out) == self.max_blocks:
                raise RuntimeError(f"chain from head {head} does not terminate (cycle)")
            out.append(idx)
            idx = self.next_ptr[idx]
        return out

    def chain_len(self, head: int) -> int:  # block_table.py:147-150
        return len(self.walk(head))

    def expand_chain(self, tail: int) -> int:  # block_table.py:152-165
        self._require(tail)
        if self.next_ptr[tail] != -1:
            raise RuntimeError(f"block {tail} is not a chain tail")
        if not self.free_list:
            raise RuntimeError("No free blocks available")
        new = self.allocate_block()
        self.next_ptr[tail] = new
        return new

    def resolve_block(self, head: int, logical: int) -> int:  # block_table.py:167-185
        row = self.walk(head)
        if logical < 0 or logical >= len(row):
            raise RuntimeError(
                f"logical block {logical} out of range for chain of {len(row)} block(s) "
                f"starting at head {head}")
        return row[logical]

    def page_table_row(self, head: int, pad_to: int | None = None) -> list[int]:
        # block_table.py:187-199
        row = self.walk(head)
        if pad_to is not None:
            if pad_to < len(row):
                raise RuntimeError(f"pad_to={pad_to} shorter than chain ({len(row)} blocks)")
            row = row + [PAD_ID] * (pad_to - len(row))
        return row

    def state(self):
        """(num_free, next_ptr, payloads, free_list) for whole-state comparison."""
        nxt = [self.next_ptr[i] if self.payload[i] is not None else -1
               for i in range(self.max_blocks)]
        return (self.num_free, nxt, [None if p is None else list(p) for p in self.payload],
                list(self.free_list))
