"""Native BlockTable: reference semantics of src/block_table.py, checked in-process.

Mirrors the behaviours the reference's own tests pin (tests/test_block_table.py,
tests/test_chain.py): lowest-id-first allocation, slot identity across cycles,
all-or-nothing chains, tail-only expansion, eager walk validation, padded rows.
"""

import numpy as np
import pytest

from src.block_table import (BLOCK_SIZE, PAD_ID, BlockTable, build_page_table,
                             build_page_table_array, resolve_block)


def test_constants():
    assert BLOCK_SIZE == 64 and PAD_ID == -1


def test_fresh_table_hands_out_lowest_ids_first():
    bt = BlockTable(max_blocks=10)
    assert [bt.allocate_block() for _ in range(3)] == [0, 1, 2]
    assert bt.num_free == 7


def test_free_is_lifo_and_reuse_gives_zeroed_payload():
    bt = BlockTable(max_blocks=4)
    a, b = bt.allocate_block(), bt.allocate_block()
    bt.get_block(a)[5] = 42
    bt.get_block(b)[5] = 99
    bt.free_block(a)
    c = bt.allocate_block()
    assert c == a                       # the freed slot comes back first
    assert bt.get_block(c) == [0] * BLOCK_SIZE
    assert bt.get_block(b)[5] == 99     # neighbour untouched


def test_payload_views_do_not_alias():
    bt = BlockTable(max_blocks=3)
    x, y = bt.allocate_block(), bt.allocate_block()
    bt.get_block(x)[0] = 111
    assert bt.get_block(y)[0] == 0
    assert bt.get_cell(x, 0) == 111
    bt.set_cell(y, 63, -7)
    assert bt.get_block(y)[63] == -7


def test_errors_match_reference_texts():
    bt = BlockTable(max_blocks=2)
    with pytest.raises(RuntimeError, match="is not allocated"):
        bt.get_block(1)
    a = bt.allocate_block()
    bt.free_block(a)
    with pytest.raises(RuntimeError, match=f"block {a} is not allocated"):
        bt.free_block(a)                # double free
    bt.allocate_block()
    bt.allocate_block()
    with pytest.raises(RuntimeError, match="No free blocks available"):
        bt.allocate_block()
    with pytest.raises(RuntimeError, match="invalid block id"):
        bt.free_block(True)
    with pytest.raises(RuntimeError, match="invalid block count"):
        bt.allocate_chain(1.5)
    with pytest.raises(RuntimeError, match="chain length must be >= 1"):
        bt.allocate_chain(0)


def test_link_and_walk():
    bt = BlockTable(max_blocks=8)
    ids = [bt.allocate_block() for _ in range(4)]
    for p, n in zip(ids, ids[1:]):
        bt.link(p, n)
    assert list(bt.walk(ids[0])) == ids
    assert bt.next_ptr[ids[-1]] == -1 and bt.next_ptr[ids[0]] == ids[1]


def test_chain_all_or_nothing():
    bt = BlockTable(max_blocks=6)
    bt.allocate_chain(2)
    before = (bt.num_free, bt.next_ptr, bt.blocks, bt.free_list)
    with pytest.raises(RuntimeError, match="insufficient free blocks: requested 5, 4 available"):
        bt.allocate_chain(5)
    assert (bt.num_free, bt.next_ptr, bt.blocks, bt.free_list) == before


def test_chain_walk_is_ascending_from_fresh_table():
    bt = BlockTable(max_blocks=16)
    h = bt.allocate_chain(3)
    assert list(bt.walk(h)) == [h, h + 1, h + 2]
    assert bt.chain_len(h) == 3 and bt.chain_tail(h) == h + 2


def test_expand_only_at_tail():
    bt = BlockTable(max_blocks=8)
    h = bt.allocate_chain(3)
    with pytest.raises(RuntimeError, match="is not a chain tail"):
        bt.expand_chain(h)
    t = bt.expand_chain(h + 2)
    assert list(bt.walk(h)) == [h, h + 1, h + 2, t]
    assert bt.next_ptr[t] == -1


def test_resolve_and_rows():
    bt = BlockTable(max_blocks=16)
    h1, h2 = bt.allocate_chain(3), bt.allocate_chain(2)
    rows = build_page_table(bt, [h1, h2], pad_to=5)
    assert rows == [[0, 1, 2, -1, -1], [3, 4, -1, -1, -1]]
    assert bt.resolve_block(h1, 2) == 2
    with pytest.raises(RuntimeError, match="out of range"):
        bt.resolve_block(h1, 3)
    with pytest.raises(RuntimeError, match="invalid logical index"):
        bt.resolve_block(h1, True)
    with pytest.raises(RuntimeError, match="shorter than chain"):
        build_page_table(bt, [h1], pad_to=2)
    assert resolve_block(rows[0], 1) == 1
    with pytest.raises(RuntimeError, match="padded"):
        resolve_block(rows[0], 3)
    with pytest.raises(RuntimeError, match="out of range"):
        resolve_block(rows[0], 5)
    with pytest.raises(RuntimeError, match="page-table row"):
        resolve_block(bt, 0)


def test_export_page_table_matches_rows_and_is_atomic():
    bt = BlockTable(max_blocks=32)
    heads = [bt.allocate_chain(n) for n in (3, 1, 5)]
    arr = build_page_table_array(bt, heads)
    assert arr.dtype == np.int32 and arr.shape == (3, 5)
    assert arr.tolist() == build_page_table(bt, heads, pad_to=5)
    buf = np.full((3, 4), 77, dtype=np.int32)
    with pytest.raises(RuntimeError, match="shorter than chain"):
        bt.export_page_table(heads, 4, out=buf)
    assert (buf == 77).all()            # nothing written on failure


def test_free_chain_releases_everything():
    bt = BlockTable(max_blocks=8)
    h = bt.allocate_chain(5)
    assert bt.free_chain(h) == 5
    assert bt.num_free == 8
    assert bt.free_list == [7, 6, 5, 0, 1, 2, 3, 4]  # freed in walk order, LIFO


def test_cycle_raises_instead_of_hanging():
    bt = BlockTable(max_blocks=4)
    h = bt.allocate_chain(3)
    bt.link(h + 2, h)
    with pytest.raises(RuntimeError, match="does not terminate"):
        bt.chain_len(h)
