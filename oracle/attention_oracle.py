"""CPU oracle for paged block attention — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
this module, and only as the checker / the timed CPU baseline. The product
path never imports it.

A numpy restatement of the reference's fp32 torch oracle ``dense_reference``
(src/kernels/block_attention.py:538-595) and of the semantics the GPU paths
add on top of it:

* :func:`dense_attention` — the full self-attention of ``dense_reference``:
  gather each sequence's scattered blocks (:571-575), half-split RoPE from
  the cos/sin tables at positions 0..T-1 (:560-564, :576-577), scores scaled
  by 1/sqrt(D) (:578), additive bias broadcast to [S, H, max_len, max_len]
  (:579-584), block mask expanded to tokens and filled with -inf (:585-592),
  softmax and PV (:593-594). Output [S, H, max_len, D], zero past seq_len.
* :func:`decode_attention` — one query row per sequence, i.e. the row of
  ``dense_reference`` whose q_cache slot holds the decoded token. The
  equivalence is pinned by tests at the shapes the full form can afford.
  Adds GQA (query head h reads KV head h // (Hq / Hkv), which is what
  ``dense_reference`` computes on K/V expanded with repeat_interleave),
  explicit query positions and the token-granular scope (Table 1 of
  src/scoping_mask.py:130-162 restated as GLOBAL tags plus the query's own
  LOCAL span).
* :func:`prefill_attention` — chunked prefill: a dense query chunk at
  absolute positions q_start..q_start+L-1 over all keys 0..q_start+L-1 with
  a causal mask, the row form of ``dense_reference`` with a (T, T) -inf
  upper-triangle bias (accepted at block_attention.py:105-108).

All arithmetic is float32 by default, like ``dense_reference``; pass
``acc=np.float64`` for a higher-precision check.
"""

from __future__ import annotations

import math

import numpy as np

BLOCK = 64
PAD_ID = -1


def _blocks_of(row, T: int, n_phys: int) -> list[int]:
    """Physical ids of the first ceil(T/64) slots (block_table.py:17-56 rules)."""
    nb = -(-T // BLOCK)
    ids = []
    for i in range(nb):
        if i >= len(row):
            raise RuntimeError(f"logical block {i} out of range for page table of {len(row)} slots")
        p = int(row[i])
        if p == PAD_ID:
            raise RuntimeError(f"logical block {i} is padded (no physical block)")
        if not (0 <= p < n_phys):
            raise RuntimeError(f"page_table entry {p} out of range for {n_phys} physical blocks")
        ids.append(p)
    return ids


def gather_tokens(cache: np.ndarray, ids: list[int], T: int, acc=np.float32) -> np.ndarray:
    """[n_phys, H, 64, D] blocks ``ids`` -> dense [H, T, D] (block_attention.py:573-575)."""
    g = cache[np.asarray(ids, dtype=np.int64)]  # [nb, H, 64, D]
    H, D = g.shape[1], g.shape[3]
    return np.ascontiguousarray(g.transpose(1, 0, 2, 3).reshape(H, -1, D)[:, :T, :]).astype(acc)


def rope_half_split(x: np.ndarray, cos_rows: np.ndarray, sin_rows: np.ndarray) -> np.ndarray:
    """(x0, x1) -> (x0 c - x1 s, x0 s + x1 c) on the two halves (block_attention.py:560-564).

    ``x`` is [..., T, D]; ``cos_rows``/``sin_rows`` are [T, D/2] and broadcast
    over the leading axes.
    """
    hf = x.shape[-1] // 2
    c = cos_rows.astype(x.dtype)
    s = sin_rows.astype(x.dtype)
    x0, x1 = x[..., :hf], x[..., hf:]
    return np.concatenate([x0 * c - x1 * s, x0 * s + x1 * c], axis=-1)


def _softmax_rows(scores: np.ndarray) -> np.ndarray:
    m = np.max(scores, axis=-1, keepdims=True)
    e = np.exp(scores - m)
    return e / np.sum(e, axis=-1, keepdims=True)


def _broadcast4(bias: np.ndarray, S: int, H: int, L: int) -> np.ndarray:
    b = bias
    while b.ndim < 4:
        b = b[None]
    return np.broadcast_to(b, (S, H, L, L))


def _broadcast_mask3(mask: np.ndarray, S: int, QB: int) -> np.ndarray:
    m = mask
    if m.ndim == 1:
        m = m[None, None, :]
    while m.ndim < 3:
        m = m[None]
    return np.broadcast_to(m, (S, QB, QB))


def dense_attention(page_table, q_cache, k_cache, v_cache, seq_lens, cos, sin,
                    bias=None, mask=None, softmax_scale=None, acc=np.float32):
    """Restatement of ``dense_reference`` (block_attention.py:538-595).

    Inputs are numpy arrays (any float dtype for the caches; they are upcast
    the way ``.float()`` does). Returns float [S, H, max_len, D].
    """
    page_table = np.asarray(page_table)
    S = page_table.shape[0]
    n_phys, H, blk, D = q_cache.shape
    lens = [int(x) for x in np.asarray(seq_lens).reshape(-1)]
    max_len = max(lens)
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D)
    qb = -(-max_len // BLOCK)
    out = np.zeros((S, H, max_len, D), dtype=acc)
    cos = np.asarray(cos, dtype=np.float32)
    sin = np.asarray(sin, dtype=np.float32)
    for s in range(S):
        T = lens[s]
        if T == 0:
            continue
        ids = _blocks_of(page_table[s], T, n_phys)
        q = rope_half_split(gather_tokens(q_cache, ids, T, acc), cos[:T], sin[:T])
        k = rope_half_split(gather_tokens(k_cache, ids, T, acc), cos[:T], sin[:T])
        v = gather_tokens(v_cache, ids, T, acc)
        scores = np.einsum("htd,hsd->hts", q, k) * acc(scale)
        if bias is not None:
            scores = scores + _broadcast4(np.asarray(bias), S, H, max_len)[s, :, :T, :T].astype(acc)
        if mask is not None:
            sc = _broadcast_mask3(np.asarray(mask), S, qb)[s]
            tok = np.repeat(np.repeat(sc, BLOCK, axis=0)[:T], BLOCK, axis=1)[:, :T]
            scores = np.where(tok == 0, -np.inf, scores)
        out[s, :, :T, :] = np.einsum("hts,hsd->htd", _softmax_rows(scores), v)
    return out


def allowed_keys(T: int, query_pos: int, *, causal: bool = False, block_mask_row=None,
                 scope_tags=None, scope_span=None) -> np.ndarray:
    """Bool [T]: which keys the query at ``query_pos`` may attend to.

    * causal: keys j <= query_pos;
    * block_mask_row: [KB] flags of the query's q-block (block_attention.py:312-316);
    * scope: Table 1 row of the query (scoping_mask.py:148-161): GLOBAL keys,
      plus keys inside the query's LOCAL span [lo, hi); a GLOBAL query has
      an empty span and itself is GLOBAL, so the diagonal is always allowed.
    """
    ok = np.ones(T, dtype=bool)
    j = np.arange(T)
    if causal:
        ok &= j <= query_pos
    if block_mask_row is not None:
        bm = np.asarray(block_mask_row).reshape(-1)
        ok &= np.repeat(bm != 0, BLOCK)[:T]
    if scope_tags is not None:
        tags = np.asarray(scope_tags).reshape(-1)[:T] != 0
        lo, hi = (0, 0) if scope_span is None else (int(scope_span[0]), int(scope_span[1]))
        ok &= tags | ((j >= lo) & (j < hi))
    return ok


def decode_attention(page_table, q, k_cache, v_cache, seq_lens, cos, sin, *, positions=None,
                     block_mask=None, scope_tags=None, scope_span=None, causal=False,
                     softmax_scale=None, acc=np.float32):
    """One decoded query per sequence over its paged keys 0..seq_len-1.

    q: [S, Hq, D]; caches [n_phys, Hkv, 64, D]; returns float [S, Hq, D].
    ``block_mask`` is [S, QB, KB] (already broadcast); the query's row is
    positions[s] // 64. ``scope_tags`` [S, >=T] uint8 (1 = GLOBAL),
    ``scope_span`` [S, 2]. A query with no allowed key returns zeros.
    """
    page_table = np.asarray(page_table)
    S, Hq, D = q.shape
    n_phys, Hkv = k_cache.shape[0], k_cache.shape[1]
    G = Hq // Hkv
    lens = [int(x) for x in np.asarray(seq_lens).reshape(-1)]
    scale = acc(softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D))
    cos = np.asarray(cos, dtype=np.float32)
    sin = np.asarray(sin, dtype=np.float32)
    out = np.zeros((S, Hq, D), dtype=acc)
    for s in range(S):
        T = lens[s]
        if T == 0:
            continue
        pos = T - 1 if positions is None else int(positions[s])
        ids = _blocks_of(page_table[s], T, n_phys)
        k = rope_half_split(gather_tokens(k_cache, ids, T, acc), cos[:T], sin[:T])  # [Hkv,T,D]
        v = gather_tokens(v_cache, ids, T, acc)
        qs = rope_half_split(q[s].astype(acc)[:, None, :], cos[pos:pos + 1], sin[pos:pos + 1])
        qs = qs.reshape(Hkv, G, D)
        scores = np.einsum("hgd,htd->hgt", qs, k) * scale
        ok = allowed_keys(
            T, pos, causal=causal,
            block_mask_row=None if block_mask is None else np.asarray(block_mask)[s, pos // BLOCK],
            scope_tags=None if scope_tags is None else np.asarray(scope_tags)[s],
            scope_span=None if scope_span is None else np.asarray(scope_span)[s])
        if not ok.any():
            continue
        scores = np.where(ok[None, None, :], scores, -np.inf)
        out[s] = np.einsum("hgt,htd->hgd", _softmax_rows(scores), v).reshape(Hq, D)
    return out


def prefill_attention(page_table, q, k_cache, v_cache, q_start, seq_lens, cos, sin, *,
                      causal=True, softmax_scale=None, acc=np.float32, scope_tags=None,
                      scope_lo=None, scope_hi=None):
    """Chunked prefill: q [S, Hq, L, D] at positions q_start[s] + i over keys 0..seq_len-1.

    Row i of sequence s attends to keys j <= q_start[s] + i when ``causal``.
    Rows with q_start[s] + i >= seq_len[s] are left zero. Token scope
    (Table 1 of scoping_mask.py:148-161, per query position): ``scope_tags``
    [S, >=T] (1 = GLOBAL key), ``scope_lo`` / ``scope_hi`` [S, >=T] the LOCAL
    span of the token at each position; key j is kept for the query at
    position i when tags[j] or lo[i] <= j < hi[i].
    """
    page_table = np.asarray(page_table)
    S, Hq, L, D = q.shape
    n_phys, Hkv = k_cache.shape[0], k_cache.shape[1]
    G = Hq // Hkv
    scale = acc(softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D))
    cos = np.asarray(cos, dtype=np.float32)
    sin = np.asarray(sin, dtype=np.float32)
    out = np.zeros((S, Hq, L, D), dtype=acc)
    for s in range(S):
        T = int(np.asarray(seq_lens).reshape(-1)[s])
        p0 = int(np.asarray(q_start).reshape(-1)[s])
        rows = max(0, min(L, T - p0))
        if rows == 0:
            continue
        ids = _blocks_of(page_table[s], T, n_phys)
        k = rope_half_split(gather_tokens(k_cache, ids, T, acc), cos[:T], sin[:T])
        v = gather_tokens(v_cache, ids, T, acc)
        qpos = np.arange(p0, p0 + rows)
        qs = rope_half_split(q[s, :, :rows].astype(acc), cos[qpos], sin[qpos])  # [Hq,rows,D]
        qs = qs.reshape(Hkv, G, rows, D)
        scores = np.einsum("hgid,htd->hgit", qs, k) * scale
        ok = np.ones((rows, T), dtype=bool)
        if causal:
            ok &= np.arange(T)[None, :] <= qpos[:, None]
        if scope_tags is not None:
            tags = np.asarray(scope_tags)[s, :T] != 0
            lo = np.asarray(scope_lo)[s, qpos][:, None]
            hi = np.asarray(scope_hi)[s, qpos][:, None]
            j = np.arange(T)[None, :]
            ok &= tags[None, :] | ((j >= lo) & (j < hi))
        scores = np.where(ok[None, None], scores, -np.inf)
        out[s, :, :rows] = np.einsum("hgit,htd->hgid", _softmax_rows(scores), v).reshape(Hq, rows, D)
    return out


def rope_tables(max_pos: int, head_dim: int, base: float = 10000.0):
    """cos/sin [max_pos, D/2]: angles in float64, rounded to float32.

    Same construction as the reference tests (tests/test_block_attention.py:293-298).
    """
    half = head_dim // 2
    inv = 1.0 / (float(base) ** (np.arange(half, dtype=np.float64) * 2.0 / head_dim))
    ang = np.arange(max_pos, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
