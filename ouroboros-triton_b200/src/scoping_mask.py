"""Table-1 scoping mask over tokens grouped into GLOBAL / LOCAL spans.

Drop-in for the reference module ``src/scoping_mask.py`` (same names, same
ValueError rules, same L x L boolean ``block_sparse_mask``), plus the compact
token-scope encoding the attention kernels consume instead of an L x L mask.

Table 1 (query i sees key j), as the reference states it (scoping_mask.py:7-25):
  * i == j                                  -> 1
  * i LOCAL,  j GLOBAL                      -> 1
  * i LOCAL,  j LOCAL in the same span      -> 1
  * i GLOBAL, j GLOBAL                      -> 1
  * i GLOBAL, j LOCAL                       -> 0
  * i LOCAL,  j LOCAL in a sibling span     -> 0

Compact encoding (no reference counterpart): per token a GLOBAL flag
(``tags``, uint8) and the [start, end) of the span holding it. Row i of
Table 1 is then ``tags[j] or start[i] <= j < end[i] (i LOCAL)``; the diagonal
is covered because a GLOBAL token carries the flag and a LOCAL token lies in
its own span. A decode kernel needs only ``tags`` and the query's span.
"""

from __future__ import annotations

from bisect import bisect_right

import numpy as np

__all__ = [
    "GLOBAL",
    "LOCAL",
    "Scope",
    "build_scope_tags",
    "same_local_scope",
    "block_sparse_mask",
    "global_rows_frozen",
    "frozen_global_rows",
    "token_scope",
    "decode_scope",
    "scope_allowed",
    "scope_bias",
    "prefill_scope",
]

GLOBAL = "global"
LOCAL = "local"


class Scope:
    """Scope names (plain strings, as in the reference)."""

    GLOBAL = "global"
    LOCAL = "local"


def _validated_sorted(spans) -> list[tuple[int, int, str]]:
    """Spans sorted by start; ValueError unless they exactly partition [0, L).

    Same rules and messages as the reference (scoping_mask.py:60-90).
    """
    cleaned: list[tuple[int, int, str]] = []
    for span in spans:
        try:
            start, end, scope = span
        except (TypeError, ValueError) as exc:
            raise ValueError(f"malformed span (want (start, end, scope)): {span!r}") from exc
        if (isinstance(start, bool) or isinstance(end, bool)
                or not isinstance(start, (int, np.integer)) or not isinstance(end, (int, np.integer))):
            raise ValueError(f"span bounds must be ints, got {span!r}")
        start, end = int(start), int(end)
        if start < 0:
            raise ValueError(f"span start must be >= 0, got {start}")
        if end <= start:
            raise ValueError(f"span must be non-empty, got ({start}, {end})")
        if scope not in (Scope.GLOBAL, Scope.LOCAL):
            raise ValueError(f"unknown scope {scope!r}; want {Scope.GLOBAL!r}/{Scope.LOCAL!r}")
        cleaned.append((start, end, scope))
    cleaned.sort()
    if cleaned and cleaned[0][0] != 0:
        raise ValueError(
            f"spans must partition starting at 0, first span starts at {cleaned[0][0]}")
    for prev, cur in zip(cleaned, cleaned[1:]):
        if cur[0] != prev[1]:
            kind = "overlap" if cur[0] < prev[1] else "gap"
            raise ValueError(f"spans do not partition [0, L): {kind} between {prev} and {cur}")
    return cleaned


def token_scope(spans):
    """Compact per-token scope: (tags uint8 [L], span_start int32 [L], span_end int32 [L])."""
    ordered = _validated_sorted(spans)
    L = ordered[-1][1] if ordered else 0
    tags = np.zeros(L, dtype=np.uint8)
    start = np.zeros(L, dtype=np.int32)
    end = np.zeros(L, dtype=np.int32)
    for s, e, sc in ordered:
        tags[s:e] = 1 if sc == Scope.GLOBAL else 0
        start[s:e] = s
        end[s:e] = e
    return tags, start, end


def decode_scope(spans, query_pos: int):
    """(tags [L], lo, hi) for one query: its row of Table 1 is ``tags[j] or lo <= j < hi``.

    A GLOBAL query gets the empty span (0, 0).
    """
    tags, start, end = token_scope(spans)
    if not (0 <= query_pos < tags.shape[0]):
        raise ValueError(f"query position {query_pos} outside the spans' extent {tags.shape[0]}")
    if tags[query_pos]:
        return tags, 0, 0
    return tags, int(start[query_pos]), int(end[query_pos])


def prefill_scope(spans_per_seq, width: int | None = None):
    """Token scope of a batch for multi-row attention (chunked prefill).

    Returns ``(tags uint8 [S, W], lo int32 [S, W], hi int32 [S, W])`` with W
    the longest extent rounded up to 16 (or ``width``): tags[s, j] = 1 for a
    GLOBAL token, and [lo, hi) the span of the token at each position. The
    query at position i keeps key j when tags[j] or lo[i] <= j < hi[i]: its
    Table-1 row (a GLOBAL query's own span holds only GLOBAL tokens).
    """
    enc = [token_scope(sp) for sp in spans_per_seq]
    longest = max((t.shape[0] for t, _, _ in enc), default=0)
    W = width if width is not None else max(16, -(-longest // 16) * 16)
    if W < longest or W % 16:
        raise ValueError(f"width {W} must be a multiple of 16 covering {longest} tokens")
    S = len(enc)
    tags = np.zeros((S, W), dtype=np.uint8)
    lo = np.zeros((S, W), dtype=np.int32)
    hi = np.zeros((S, W), dtype=np.int32)
    for s, (t, a, b) in enumerate(enc):
        tags[s, : t.shape[0]] = t
        lo[s, : t.shape[0]] = a
        hi[s, : t.shape[0]] = b
    return tags, lo, hi


def scope_allowed(spans) -> np.ndarray:
    """Full Table-1 mask as a bool [L, L] array, built from the compact encoding."""
    tags, start, end = token_scope(spans)
    L = tags.shape[0]
    j = np.arange(L)
    local_row = (tags == 0)[:, None]
    in_span = (j[None, :] >= start[:, None]) & (j[None, :] < end[:, None])
    return (tags != 0)[None, :] | (local_row & in_span) | np.eye(L, dtype=bool)


def scope_bias(spans, dtype=np.float32) -> np.ndarray:
    """Additive bias [L, L]: 0 where Table 1 allows, -inf elsewhere."""
    return np.where(scope_allowed(spans), 0.0, -np.inf).astype(dtype)


def build_scope_tags(spans) -> list[str]:
    """Per-token scope names, length L (reference scoping_mask.py:93-111)."""
    tags: list[str] = []
    for start, end, scope in _validated_sorted(spans):
        tags.extend([scope] * (end - start))
    return tags


def same_local_scope(i: int, j: int, spans) -> bool:
    """True iff tokens i and j lie in one LOCAL span (reference scoping_mask.py:114-127)."""
    ordered = _validated_sorted(spans)
    starts = [s for s, _, _ in ordered]

    def owner(tok: int):
        k = bisect_right(starts, tok) - 1
        if k < 0:
            return None
        s, e, sc = ordered[k]
        return (s, e) if (s <= tok < e and sc == Scope.LOCAL) else None

    oi, oj = owner(i), owner(j)
    return oi is not None and oi == oj


def block_sparse_mask(spans) -> list[list[bool]]:
    """L x L boolean mask implementing Table 1 (reference scoping_mask.py:130-162)."""
    if not _validated_sorted(spans):
        return []
    return scope_allowed(spans).tolist()


def global_rows_frozen(mask_before, mask_after, spans_after) -> bool:
    """Did every GLOBAL row survive an [EXPAND] unchanged? Never raises.

    Reference semantics (scoping_mask.py:165-190): a row tagged GLOBAL under
    ``spans_after`` must equal its ``mask_before`` row over the old extent and
    be False beyond it; any malformed input reads as False.
    """
    try:
        ordered = _validated_sorted(spans_after)
        total_new = ordered[-1][1] if ordered else 0
        total_old = len(mask_before)
        if total_new < total_old or len(mask_after) != total_new:
            return False
        if any(len(r) != total_new for r in mask_after):
            return False
        for s, e, sc in ordered:
            if sc != Scope.GLOBAL:
                continue
            for i in range(s, e):
                expected = list(mask_before[i]) + [False] * (total_new - total_old)
                if list(mask_after[i]) != expected:
                    return False
        return True
    except (TypeError, ValueError, IndexError):
        return False


frozen_global_rows = global_rows_frozen
