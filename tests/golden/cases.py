"""Seeded input builders shared by the golden-fixture script and the tests.

``make_golden.py`` runs these against the reference's own ``src`` package
(its BlockTable, its dense_reference); the tests run them against this
repository's ``src`` package and compare with the recorded outputs. The
random draws come from ``torch.Generator`` on the CPU and ``random.Random``,
so both sides see identical inputs for a given seed.

Block placement recipe for every case: allocate the whole pool, free it in a
seeded shuffled order, then ``allocate_chain(ceil(len / 64))`` per sequence,
which scatters each chain across the pool in a deterministic order.
"""

from __future__ import annotations

import math
import random

BLOCK = 64


def scattered_chains(block_table_cls, pool: int, lens, seed: int):
    """(table, heads, page_table rows padded to max_b) under the placement recipe."""
    bt = block_table_cls(max_blocks=pool)
    ids = [bt.allocate_block() for _ in range(pool)]
    random.Random(seed).shuffle(ids)
    for i in ids:
        bt.free_block(i)
    heads = [bt.allocate_chain(max(1, -(-int(n) // BLOCK))) for n in lens]
    max_b = max(max(1, -(-int(n) // BLOCK)) for n in lens)
    rows = [list(bt.page_table_row(h, pad_to=max_b)) for h in heads]
    return bt, heads, rows


def rope_tables_torch(torch, max_pos: int, head_dim: int, base: float):
    """cos/sin [max_pos, D/2], float64 angles rounded to float32."""
    half = head_dim // 2
    inv = 1.0 / (float(base) ** (torch.arange(half, dtype=torch.float64) * 2.0 / head_dim))
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cos(ang).float(), torch.sin(ang).float()


def paged_caches(torch, seed: int, n_phys: int, heads: int, head_dim: int, std: float,
                 dtype, with_q: bool = True):
    """q/k/v caches [n_phys, heads, 64, D] ~ std * N(0, 1), drawn in q, k, v order."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    shape = (n_phys, heads, BLOCK, head_dim)
    out = []
    for _ in range(3 if with_q else 2):
        out.append((torch.randn(shape, generator=g) * std).to(dtype))
    return out


def config1_case(torch, block_table_cls, seed: int = 1):
    """CPU-runnable decode case: 4 seqs, lens {64,130,200,511}, H=8, D=64, pool 64, fp32."""
    lens = [64, 130, 200, 511]
    bt, heads, rows = scattered_chains(block_table_cls, 64, lens, seed)
    q, k, v = paged_caches(torch, seed, 64, 8, 64, 1.0, torch.float32)
    cos, sin = rope_tables_torch(torch, len(rows[0]) * BLOCK, 64, 10000.0)
    return dict(lens=lens, rows=rows, q_cache=q, k_cache=k, v_cache=v, cos=cos, sin=sin)


def small_full_case(torch, block_table_cls, seed: int, dtype=None, lens=(192, 150),
                    num_heads=2, head_dim=32):
    """The reference's GPU-test shape (2 seqs x 3 blocks, H=2, D=32) under the recipe."""
    dtype = torch.float32 if dtype is None else dtype
    bt, heads, rows = scattered_chains(block_table_cls, 16, lens, seed)
    q, k, v = paged_caches(torch, seed, 16, num_heads, head_dim, 1.0, dtype)
    cos, sin = rope_tables_torch(torch, len(rows[0]) * BLOCK, head_dim, 10000.0)
    return dict(lens=list(lens), rows=rows, q_cache=q, k_cache=k, v_cache=v, cos=cos, sin=sin)


def segment_spans(length: int, seed: int, lo: int = 32, hi: int = 512, p_local: float = 0.5):
    """Per-sequence random segments covering [0, length).

    Segment lengths are uniform in [lo, hi] (the last one truncated); segment
    0 is GLOBAL, later segments are LOCAL with probability ``p_local``.
    """
    rng = random.Random(seed)
    spans, start, idx = [], 0, 0
    while start < length:
        n = min(rng.randint(lo, hi), length - start)
        tag = "global" if idx == 0 or rng.random() >= p_local else "local"
        spans.append((start, start + n, tag))
        start += n
        idx += 1
    return spans


def input_checksum(t) -> list[float]:
    """(sum, sum of squares) in float64 — detects generator drift across machines."""
    x = t.double()
    return [float(x.sum()), float((x * x).sum())]


def config2_slice_case(torch, block_table_cls, seed: int = 2, lens=(700, 1500)):
    """Two sequences of the fp16 MHA decode shape (H=32, D=128, 0.5*N(0,1), base 1e4)."""
    pool = 64
    bt, heads, rows = scattered_chains(block_table_cls, pool, lens, seed)
    q, k, v = paged_caches(torch, seed, pool, 32, 128, 0.5, torch.float16)
    cos, sin = rope_tables_torch(torch, len(rows[0]) * BLOCK, 128, 10000.0)
    spans = [segment_spans(n, seed * 1000 + i) for i, n in enumerate(lens)]
    return dict(lens=list(lens), rows=rows, q_cache=q, k_cache=k, v_cache=v, cos=cos, sin=sin,
                spans=spans)


def gqa_decode_case(torch, block_table_cls, seed: int = 3, lens=(333, 64, 1025),
                    hq=16, hkv=2, head_dim=128, dtype=None, base=500000.0):
    """Small GQA decode case (group 8), bf16 0.5*N(0,1), RoPE base 5e5."""
    dtype = torch.bfloat16 if dtype is None else dtype
    pool = 48
    bt, heads, rows = scattered_chains(block_table_cls, pool, lens, seed)
    k, v = paged_caches(torch, seed, pool, hkv, head_dim, 0.5, dtype, with_q=False)
    g = torch.Generator(device="cpu").manual_seed(seed + 7)
    q = (torch.randn((len(lens), hq, head_dim), generator=g) * 0.5).to(dtype)
    cos, sin = rope_tables_torch(torch, len(rows[0]) * BLOCK, head_dim, base)
    return dict(lens=list(lens), rows=rows, q=q, k_cache=k, v_cache=v, cos=cos, sin=sin)


def alloc_script(seed: int, max_blocks: int = 24, n_ops: int = 300):
    """A seeded op script that never links a cycle.

    Ops: alloc, free, chain, expand, link (only a tail onto the head of a
    different chain, never creating a cycle), walk, len, resolve, row,
    set/get cell, and deliberate error cases (double free, bad ids, zero or
    oversized chains, expand on a non-tail).
    """
    rng = random.Random(seed)
    ops = []
    for _ in range(n_ops):
        kind = rng.choice(["alloc", "free", "chain", "expand", "link", "walk", "len",
                           "resolve", "row", "cell", "bad"])
        if kind == "alloc":
            ops.append(["alloc"])
        elif kind == "free":
            ops.append(["free", rng.randrange(-2, max_blocks + 2)])
        elif kind == "chain":
            ops.append(["chain", rng.randrange(-1, max_blocks // 2)])
        elif kind == "expand":
            ops.append(["expand", rng.randrange(0, max_blocks)])
        elif kind == "link":
            ops.append(["link", rng.randrange(0, max_blocks), rng.randrange(0, max_blocks)])
        elif kind == "walk":
            ops.append(["walk", rng.randrange(0, max_blocks)])
        elif kind == "len":
            ops.append(["len", rng.randrange(0, max_blocks)])
        elif kind == "resolve":
            ops.append(["resolve", rng.randrange(0, max_blocks), rng.randrange(-1, 6)])
        elif kind == "row":
            ops.append(["row", rng.randrange(0, max_blocks), rng.choice([None, 0, 3, 8, 16])])
        elif kind == "cell":
            ops.append(["cell", rng.randrange(0, max_blocks), rng.randrange(0, BLOCK),
                        rng.randrange(-1000, 1000)])
        else:
            ops.append(["free", rng.randrange(0, max_blocks)])
    return ops


def link_is_safe(next_of, allocated, a: int, b: int) -> bool:
    """True when linking a -> b keeps every chain acyclic and a is a tail."""
    if a not in allocated or b not in allocated or a == b:
        return False
    if next_of(a) != -1:
        return False
    # b's chain must not reach a
    seen, cur = 0, b
    while cur != -1 and seen <= len(allocated):
        if cur == a:
            return False
        cur = next_of(cur)
        seen += 1
    return True


def mean_abs(x) -> float:
    n = x.numel()
    return float(x.abs().sum()) / max(n, 1)


def isqrt_scale(d: int) -> float:
    return 1.0 / math.sqrt(d)
