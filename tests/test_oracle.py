"""The CPU oracle, pinned against outputs of the reference itself.

tests/golden/*.npz were produced by the reference's dense_reference (torch
fp32) and golden_attention_mt (pure Python) on seeded inputs
(tests/golden/make_golden.py). The numpy restatement in oracle/ must
reproduce them before it is trusted as the checker of the CUDA kernels.
"""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

import cases
from oracle import attention_oracle as ao
from src.block_table import BlockTable
from src.scoping_mask import decode_scope, scope_bias

GOLD = Path(__file__).resolve().parent / "golden"


def _np(t):
    return t.float().numpy() if t.dtype in (torch.float16, torch.bfloat16) else t.numpy()


def test_config1_inputs_and_page_table_are_reproduced():
    g = np.load(GOLD / "decode_c1.npz")
    c = cases.config1_case(torch, BlockTable, seed=1)
    assert np.asarray(c["rows"]).tolist() == g["rows"].tolist()   # allocator bit-exact
    assert np.allclose(cases.input_checksum(c["q_cache"]), g["qsum"], rtol=1e-12)
    assert np.allclose(cases.input_checksum(c["k_cache"]), g["ksum"], rtol=1e-12)


def test_dense_restatement_matches_reference_rows_config1():
    g = np.load(GOLD / "decode_c1.npz")
    c = cases.config1_case(torch, BlockTable, seed=1)
    out = ao.dense_attention(np.asarray(c["rows"]), _np(c["q_cache"]), _np(c["k_cache"]),
                             _np(c["v_cache"]), c["lens"], _np(c["cos"]), _np(c["sin"]))
    lens = c["lens"]
    dec = np.stack([out[s, :, lens[s] - 1] for s in range(4)])
    assert np.abs(dec - g["decode"]).max() < 2e-5
    probes = np.stack([out[3, :, r] for r in g["probe_rows"]])
    assert np.abs(probes - g["probes"]).max() < 2e-5


def test_decode_restatement_equals_dense_row_config1():
    g = np.load(GOLD / "decode_c1.npz")
    c = cases.config1_case(torch, BlockTable, seed=1)
    rows, lens = np.asarray(c["rows"]), c["lens"]
    q = np.stack([_np(c["q_cache"])[rows[s][(lens[s] - 1) // 64], :, (lens[s] - 1) % 64]
                  for s in range(4)])
    dec = ao.decode_attention(rows, q, _np(c["k_cache"]), _np(c["v_cache"]), lens,
                              _np(c["cos"]), _np(c["sin"]))
    assert np.abs(dec - g["decode"]).max() < 2e-5


@pytest.mark.parametrize("name", ["bm", "plain", "f16"])
def test_dense_restatement_matches_reference_small(name):
    g = np.load(GOLD / "attn_small.npz")
    seed = {"bm": 1234, "plain": 77, "f16": 5}[name]
    dt = torch.float16 if name == "f16" else torch.float32
    c = cases.small_full_case(torch, BlockTable, seed, dtype=dt)
    assert np.asarray(c["rows"]).tolist() == g[f"{name}_rows"].tolist()
    kw = {}
    if name == "bm":
        gen = torch.Generator().manual_seed(seed + 1)
        bias = torch.randn(1, 2, max(c["lens"]), max(c["lens"]), generator=gen) * 0.25
        scope = torch.randint(0, 2, (2, 3, 3), generator=gen) | torch.eye(3, dtype=torch.int64)
        assert np.allclose(cases.input_checksum(bias), g["bm_biassum"], rtol=1e-12)
        assert scope.to(torch.int8).numpy().tolist() == g["bm_mask"].tolist()
        kw = dict(bias=bias.numpy(), mask=scope.numpy())
    out = ao.dense_attention(np.asarray(c["rows"]), _np(c["q_cache"]), _np(c["k_cache"]),
                             _np(c["v_cache"]), c["lens"], _np(c["cos"]), _np(c["sin"]), **kw)
    assert np.abs(out - g[f"{name}_out"]).max() < 2e-5


def test_decode_restatement_with_scope_matches_reference_c2_slice():
    g = np.load(GOLD / "decode_c2s.npz")
    c = cases.config2_slice_case(torch, BlockTable)
    assert np.asarray(c["rows"]).tolist() == g["rows"].tolist()
    spans = json.loads(str(g["spans"]))
    assert [[list(x) for x in sp] for sp in c["spans"]] == spans
    rows, lens = np.asarray(c["rows"]), c["lens"]
    qc = _np(c["q_cache"])
    q = np.stack([qc[rows[s][(lens[s] - 1) // 64], :, (lens[s] - 1) % 64] for s in range(2)])
    tags = np.zeros((2, max(lens)), np.uint8)
    span = np.zeros((2, 2), np.int32)
    for s in range(2):
        t, lo, hi = decode_scope([tuple(x) for x in spans[s]], lens[s] - 1)
        tags[s, :lens[s]] = t
        span[s] = (lo, hi)
    dec = ao.decode_attention(rows, q, _np(c["k_cache"]), _np(c["v_cache"]), lens,
                              _np(c["cos"]), _np(c["sin"]), scope_tags=tags, scope_span=span)
    assert np.abs(dec - g["decode"]).max() < 2e-5
    # the same through the full-mask path: dense restatement with a -inf bias
    bias = np.full((2, 1, max(lens), max(lens)), -np.inf, np.float32)
    for s in range(2):
        bias[s, 0, :lens[s], :lens[s]] = scope_bias([tuple(x) for x in spans[s]])
    full = ao.dense_attention(rows, qc, _np(c["k_cache"]), _np(c["v_cache"]), lens,
                              _np(c["cos"]), _np(c["sin"]), bias=bias)
    assert np.abs(np.stack([full[s, :, lens[s] - 1] for s in range(2)]) - g["decode"]).max() < 2e-5


def test_decode_restatement_gqa_matches_reference():
    g = np.load(GOLD / "decode_gqa.npz")
    c = cases.gqa_decode_case(torch, BlockTable)
    assert np.asarray(c["rows"]).tolist() == g["rows"].tolist()
    dec = ao.decode_attention(np.asarray(c["rows"]), _np(c["q"]), _np(c["k_cache"]),
                              _np(c["v_cache"]), c["lens"], _np(c["cos"]), _np(c["sin"]))
    assert np.abs(dec - g["decode"]).max() < 2e-5


@pytest.mark.parametrize("d", [8, 32])
def test_restatement_matches_golden_attention_mt(d):
    """golden_attention_mt is interleaved-pair RoPE; the engine layout is half-split.

    Payloads and outputs are moved between the two with the channel
    permutation perm(t) = (t % 2) * (d/2) + t // 2 (reference_attention.py:141-213).
    """
    g = np.load(GOLD / "golden_mt.npz")
    pay, ids = g[f"d{d}_payload"], g[f"d{d}_ids"]
    perm = np.array([(t % 2) * (d // 2) + t // 2 for t in range(d)])
    n_phys = int(ids.max()) + 1
    caches = np.zeros((3, n_phys, 1, 64, d), np.float32)
    for bi, pid in enumerate(ids):
        for ci in range(3):
            caches[ci, pid, 0][:, perm] = pay[bi, ci]
    half = d // 2
    inv = np.array([10000.0 ** (-2.0 * t / d) for t in range(half)])
    ang = np.arange(256)[:, None] * inv[None, :]
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    rows, lens = g[f"d{d}_rows"], g[f"d{d}_lens"]
    qpos = json.loads(str(g[f"d{d}_qpos"]))
    got = []
    for s, plist in enumerate(qpos):
        for p in plist:
            blk, slot = rows[s][p // 64], p % 64
            q = caches[0, blk, :, slot][None]          # [1, 1, d]
            o = ao.decode_attention(rows[s:s + 1], q, caches[1], caches[2], [int(lens[s])],
                                    cos, sin, positions=[p], acc=np.float64)
            got.append(o[0, 0])
    gold_perm = np.zeros_like(g[f"d{d}_gold"])
    gold_perm[:, perm] = g[f"d{d}_gold"]
    assert np.abs(np.stack(got) - gold_perm).max() < 1e-5


def test_prefill_restatement_equals_dense_rows_with_causal_bias():
    c = cases.small_full_case(torch, BlockTable, 11, lens=(192, 150), num_heads=2, head_dim=32)
    rows, lens = np.asarray(c["rows"]), c["lens"]
    qc, kc, vc = _np(c["q_cache"]), _np(c["k_cache"]), _np(c["v_cache"])
    cos, sin = _np(c["cos"]), _np(c["sin"])
    L = max(lens)
    causal = np.where(np.tril(np.ones((L, L), bool)), 0.0, -np.inf).astype(np.float32)
    full = ao.dense_attention(rows, qc, kc, vc, lens, cos, sin, bias=causal)
    # chunk = tokens [64, 150) of each sequence, queries taken from the q cache
    q = np.zeros((2, 2, 86, 32), np.float32)
    for s in range(2):
        for i in range(86):
            p = 64 + i
            if p < lens[s]:
                q[s, :, i] = qc[rows[s][p // 64], :, p % 64]
    got = ao.prefill_attention(rows, q, kc, vc, [64, 64], lens, cos, sin, causal=True)
    for s in range(2):
        n = min(86, lens[s] - 64)
        assert np.abs(got[s, :, :n] - full[s, :, 64:64 + n]).max() < 2e-5


def test_prefill_restatement_with_scope_equals_dense_rows_with_table1_bias():
    """Scoped prefill rows (tags / per-position spans) equal the dense restatement
    with the Table-1 mask of scoping_mask plus causality as an additive bias."""
    from src.scoping_mask import prefill_scope, scope_bias

    c = cases.small_full_case(torch, BlockTable, 13, lens=(192, 150), num_heads=2, head_dim=32)
    rows, lens = np.asarray(c["rows"]), c["lens"]
    qc, kc, vc = _np(c["q_cache"]), _np(c["k_cache"]), _np(c["v_cache"])
    cos, sin = _np(c["cos"]), _np(c["sin"])
    spans = [[(0, 40, "global"), (40, 100, "local"), (100, 130, "global"), (130, 192, "local")],
             [(0, 70, "local"), (70, 90, "global"), (90, 150, "local")]]
    tags, lo, hi = prefill_scope(spans)
    L = max(lens)
    bias = np.full((2, 1, L, L), -np.inf, np.float32)
    for s in range(2):
        n = lens[s]
        b = scope_bias(spans[s]) + np.where(np.tril(np.ones((n, n), bool)), 0.0, -np.inf)
        bias[s, 0, :n, :n] = b
    full = ao.dense_attention(rows, qc, kc, vc, lens, cos, sin, bias=bias)
    q = np.zeros((2, 2, 86, 32), np.float32)
    for s in range(2):
        for i in range(86):
            p = 64 + i
            if p < lens[s]:
                q[s, :, i] = qc[rows[s][p // 64], :, p % 64]
    got = ao.prefill_attention(rows, q, kc, vc, [64, 64], lens, cos, sin, causal=True,
                               scope_tags=tags, scope_lo=lo, scope_hi=hi)
    for s in range(2):
        n = min(86, lens[s] - 64)
        assert np.abs(got[s, :, :n] - full[s, :, 64:64 + n]).max() < 2e-5


def test_prefill_scope_arrays_follow_token_scope():
    from src.scoping_mask import prefill_scope, token_scope

    spans = [[(0, 5, "local"), (5, 9, "global")], [(0, 20, "global")]]
    tags, lo, hi = prefill_scope(spans)
    assert tags.shape == (2, 32) and tags.dtype == np.uint8 and lo.dtype == np.int32
    for s, sp in enumerate(spans):
        t, a, b = token_scope(sp)
        n = t.shape[0]
        assert (tags[s, :n] == t).all() and (lo[s, :n] == a).all() and (hi[s, :n] == b).all()
        assert not tags[s, n:].any()
    with pytest.raises(ValueError):
        prefill_scope(spans, width=24)
