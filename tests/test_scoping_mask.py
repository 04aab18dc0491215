"""Table-1 scope: the drop-in helpers and the compact encoding the kernels use.

The reference pins its mask with a hand-written 8-token literal
(tests/test_scoping_mask.py:38-52); here the same 8-token case is rebuilt
from the Table-1 rules by hand (rows by scope class), and 12 seeded span sets
recorded from the reference's block_sparse_mask (tests/golden/scope_masks.json)
are compared cell by cell.
"""

import json
from pathlib import Path

import numpy as np
import pytest

from src.scoping_mask import (GLOBAL, LOCAL, Scope, block_sparse_mask, build_scope_tags,
                              decode_scope, global_rows_frozen, same_local_scope, scope_allowed,
                              scope_bias, token_scope)

G, L = "global", "local"
SPANS = [(0, 2, G), (2, 5, L), (5, 8, L)]   # G G | A A A | B B B
GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "scope_masks.json").read_text())


def _hand_mask():
    # Table 1 by scope class: GLOBAL rows see only GLOBAL keys; a LOCAL row
    # sees GLOBAL keys and its own span.
    glob = [1, 1, 0, 0, 0, 0, 0, 0]
    span_a = [1, 1, 1, 1, 1, 0, 0, 0]
    span_b = [1, 1, 0, 0, 0, 1, 1, 1]
    rows = [glob, glob, span_a, span_a, span_a, span_b, span_b, span_b]
    return [[bool(v) for v in r] for r in rows]


def test_scope_names():
    assert Scope.GLOBAL == GLOBAL == "global" and Scope.LOCAL == LOCAL == "local"


def test_eight_token_table1_by_hand():
    assert block_sparse_mask(SPANS) == _hand_mask()
    m = block_sparse_mask(SPANS)
    assert all(isinstance(v, bool) for r in m for v in r)
    assert m[2][0] and not m[0][2]          # deliberate asymmetry


@pytest.mark.parametrize("case", GOLDEN, ids=[f"L{len(c['mask'])}" for c in GOLDEN])
def test_matches_reference_block_sparse_mask(case):
    spans = [tuple(s) for s in case["spans"]]
    want = [[c == "1" for c in row] for row in case["mask"]]
    assert block_sparse_mask(spans) == want
    tags, start, end = token_scope(spans)
    for i in range(len(want)):
        _, lo, hi = decode_scope(spans, i)
        j = np.arange(len(want))
        row = (tags != 0) | ((j >= lo) & (j < hi))
        assert row.tolist() == want[i]      # compact encoding reproduces every row


def test_tags_and_partition_errors():
    assert build_scope_tags([(2, 5, L), (5, 8, L), (0, 2, G)]) == [G, G] + [L] * 6
    assert build_scope_tags([]) == [] and block_sparse_mask([]) == []
    for bad in ([(0, 2, G), (3, 5, L)], [(0, 3, G), (2, 5, L)], [(1, 4, L)], [(0, 0, G)],
                [(-1, 2, G)], [(0, 4, "friend")], [(0, 2)], [(0.0, 2, G)]):
        with pytest.raises(ValueError):
            build_scope_tags(bad)


def test_same_local_scope():
    assert same_local_scope(2, 4, SPANS) and same_local_scope(3, 3, SPANS)
    assert not same_local_scope(2, 6, SPANS) and not same_local_scope(0, 1, SPANS)
    assert not same_local_scope(-1, 2, SPANS) and not same_local_scope(0, 0, [])


def test_global_rows_frozen():
    before = block_sparse_mask(SPANS)
    grown = SPANS[:-1] + [(5, 10, L)]
    after = block_sparse_mask(grown)
    assert global_rows_frozen(before, after, grown)
    broken = [list(r) for r in after]
    broken[0][3] = True
    assert not global_rows_frozen(before, broken, grown)
    assert not global_rows_frozen(before, after, [(0, 1, G)])
    assert not global_rows_frozen(before, after, "garbage")


def test_bias_and_allowed_agree():
    a = scope_allowed(SPANS)
    b = scope_bias(SPANS)
    assert ((b == 0) == a).all() and np.isneginf(b[~a]).all()
    tags, lo, hi = decode_scope(SPANS, 0)
    assert (lo, hi) == (0, 0) and tags.tolist() == [1, 1, 0, 0, 0, 0, 0, 0]
    assert decode_scope(SPANS, 6)[1:] == (5, 8)
