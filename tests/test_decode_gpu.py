"""Paged decode on the GPU vs the oracle and the reference's recorded outputs.

Tolerances: fp16/bf16 max-abs 2e-2 and mean-abs 2e-3 against
the fp32 oracle; fp32 caches (CUDA-core path, fp32 math) 1e-4 max-abs.
"""

import json
import random
from pathlib import Path

import numpy as np
import pytest
import torch

import cases
from oracle import attention_oracle as ao
from src.block_table import BlockTable, build_page_table_array
from src.kernels import block_attention as ba
from src.scoping_mask import decode_scope

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"
HALF_MAX, HALF_MEAN = 2e-2, 2e-3


def _np(t):
    t = t.detach().cpu()
    return (t.float() if t.dtype in (torch.float16, torch.bfloat16) else t).numpy()


def _close_half(got, want, label):
    err = np.abs(_np(got).astype(np.float64) - np.asarray(want, np.float64))
    assert err.max() <= HALF_MAX and err.mean() <= HALF_MEAN, (
        f"{label}: max-abs {err.max():.3e}, mean-abs {err.mean():.3e}")


def _random_case(seed, lens, hq, hkv, d, dtype, pool=None, base=500000.0, dev="cuda"):
    rng = random.Random(seed)
    need = sum(max(1, -(-n // 64)) for n in lens)
    pool = pool or need + 7
    bt = BlockTable(pool)
    ids = [bt.allocate_block() for _ in range(pool)]
    rng.shuffle(ids)
    for i in ids:
        bt.free_block(i)
    heads = [bt.allocate_chain(max(1, -(-n // 64))) for n in lens]
    pt = build_page_table_array(bt, heads)
    g = torch.Generator().manual_seed(seed)
    k = (torch.randn(pool, hkv, 64, d, generator=g) * 0.5).to(dtype)
    v = (torch.randn(pool, hkv, 64, d, generator=g) * 0.5).to(dtype)
    q = (torch.randn(len(lens), hq, d, generator=g) * 0.5).to(dtype)
    cos, sin = ao.rope_tables(pt.shape[1] * 64, d, base)
    return dict(pt=pt, q=q, k=k, v=v, lens=np.asarray(lens, np.int32), cos=cos, sin=sin)


def _run(c, **kw):
    return ba.block_attention_decode(torch.from_numpy(c["pt"]).cuda(), c["q"].cuda(),
                                     c["k"].cuda(), c["v"].cuda(),
                                     torch.from_numpy(c["lens"]).cuda(),
                                     torch.from_numpy(c["cos"]).cuda(),
                                     torch.from_numpy(c["sin"]).cuda(), **kw)


def _oracle(c, **kw):
    return ao.decode_attention(c["pt"], _np(c["q"]), _np(c["k"]), _np(c["v"]), c["lens"],
                               c["cos"], c["sin"], **kw)


def test_config1_fp32_matches_reference_rows(cuda):
    g = np.load(GOLD / "decode_c1.npz")
    c = cases.config1_case(torch, BlockTable, seed=1)
    rows, lens = np.asarray(c["rows"]), c["lens"]
    q = torch.stack([c["q_cache"][rows[s][(lens[s] - 1) // 64], :, (lens[s] - 1) % 64]
                     for s in range(4)])
    for split in (0, 1, 3):
        out = ba.block_attention_decode(torch.from_numpy(rows).cuda(), q.cuda(),
                                        c["k_cache"].cuda(), c["v_cache"].cuda(),
                                        torch.tensor(lens).cuda(), c["cos"].cuda(),
                                        c["sin"].cuda(), split_blocks=split)
        assert np.abs(_np(out) - g["decode"]).max() < 1e-4, split


def test_fp32_has_no_tensor_core_build(cuda):
    c = _random_case(1, [100], 8, 8, 64, torch.float32)
    with pytest.raises(RuntimeError, match="tensor-core decode not built"):
        _run(c, kernel="tc")


@pytest.mark.parametrize("kernel", ["tc", "simt"])
@pytest.mark.parametrize("split", [0, 1, 2, 5])
def test_gqa_bf16_matches_reference(cuda, kernel, split):
    g = np.load(GOLD / "decode_gqa.npz")
    c = cases.gqa_decode_case(torch, BlockTable)
    out = ba.block_attention_decode(torch.tensor(c["rows"], dtype=torch.int32).cuda(),
                                    c["q"].cuda(), c["k_cache"].cuda(), c["v_cache"].cuda(),
                                    torch.tensor(c["lens"]).cuda(), c["cos"].cuda(),
                                    c["sin"].cuda(), kernel=kernel, split_blocks=split)
    _close_half(out, g["decode"], f"gqa {kernel} split={split}")


@pytest.mark.parametrize("kernel", ["tc", "simt"])
def test_config2_slice_scope_fp16_matches_reference(cuda, kernel):
    g = np.load(GOLD / "decode_c2s.npz")
    c = cases.config2_slice_case(torch, BlockTable)
    spans = json.loads(str(g["spans"]))
    rows, lens = np.asarray(c["rows"]), c["lens"]
    q = torch.stack([c["q_cache"][rows[s][(lens[s] - 1) // 64], :, (lens[s] - 1) % 64]
                     for s in range(2)])
    tags = torch.zeros(2, max(lens), dtype=torch.uint8)
    span = torch.zeros(2, 2, dtype=torch.int32)
    for s in range(2):
        t, lo, hi = decode_scope([tuple(x) for x in spans[s]], lens[s] - 1)
        tags[s, :lens[s]] = torch.from_numpy(t)
        span[s] = torch.tensor([lo, hi])
    out = ba.block_attention_decode(torch.from_numpy(rows).cuda(), q.cuda(),
                                    c["k_cache"].cuda(), c["v_cache"].cuda(),
                                    torch.tensor(lens).cuda(), c["cos"].cuda(), c["sin"].cuda(),
                                    scope=(tags, span), kernel=kernel, split_blocks=4)
    _close_half(out, g["decode"], f"config-2 slice {kernel}")


@pytest.mark.parametrize("hq,hkv,d,dtype", [
    (64, 8, 128, torch.bfloat16),   # Llama-3-70B attention shape
    (32, 8, 128, torch.bfloat16),   # Llama-3-8B shape
    (32, 32, 128, torch.float16),   # MHA
    (16, 16, 64, torch.float16),
    (12, 6, 64, torch.bfloat16),    # KV heads not a multiple of 8
    (8, 4, 128, torch.float16),     # 4 KV heads per CTA (one TMA box covers 4 heads)
    (3, 1, 64, torch.bfloat16),     # one KV head, odd GQA group
])
def test_random_shapes_vs_oracle(cuda, hq, hkv, d, dtype):
    lens = [1, 63, 64, 65, 700, 2049, 1500, 129]
    c = _random_case(hq * 7 + d, lens, hq, hkv, d, dtype)
    want = _oracle(c)
    for kernel in ("auto", "simt"):
        for split in (0, 3, 32):
            _close_half(_run(c, kernel=kernel, split_blocks=split), want,
                        f"{hq}/{hkv}/{d} {kernel} split={split}")


@pytest.mark.parametrize("hq,hkv,d,dtype", [
    (16, 8, 128, torch.bfloat16),   # combine with 16-byte column loads
    (4, 2, 34, torch.float16),      # head_dim not a multiple of 4: one column per lane
])
def test_more_than_32_splits_vs_oracle(cuda, hq, hkv, d, dtype):
    """One block per split: 2049 tokens give 33 partials per row, so the combine
    walks its splits in more than one pass of 32."""
    lens = [2049, 2200, 70, 1]
    c = _random_case(hq * 3 + d, lens, hq, hkv, d, dtype)
    want = _oracle(c)
    for kernel in ("auto", "simt"):
        _close_half(_run(c, kernel=kernel, split_blocks=1), want,
                    f"{hq}/{hkv}/{d} {kernel} split=1")


def test_positions_causal_and_block_mask(cuda):
    lens = [900, 300, 1300, 64]
    c = _random_case(5, lens, 16, 2, 128, torch.bfloat16)
    pos = np.array([500, 299, 70, 10], np.int32)
    S, mb = c["pt"].shape
    bm = np.ones((S, mb, mb), np.int8)
    bm[0, 500 // 64, 2] = 0
    bm[2, 70 // 64, 0] = 0
    want = _oracle(c, positions=pos, causal=True, block_mask=bm)
    for kernel in ("tc", "simt"):
        out = _run(c, positions=torch.from_numpy(pos).cuda(), causal=True,
                   mask=torch.from_numpy(bm).cuda(), kernel=kernel, split_blocks=2)
        _close_half(out, want, f"positions/causal/mask {kernel}")
    # non-causal with explicit positions: all keys, RoPE at the given position
    want = _oracle(c, positions=pos)
    _close_half(_run(c, positions=torch.from_numpy(pos).cuda()), want, "positions")


def test_empty_and_fully_masked_rows_are_zero(cuda):
    c = _random_case(9, [0, 200, 130], 8, 1, 128, torch.bfloat16)
    c["pt"][0, :] = -1                          # an empty sequence owns no block
    S, mb = c["pt"].shape
    bm = np.ones((S, mb, mb), np.int8)
    bm[2] = 0                                   # sequence 2 sees nothing
    for kernel in ("tc", "simt"):
        out = _np(_run(c, mask=torch.from_numpy(bm).cuda(), kernel=kernel))
        assert (out[0] == 0).all() and (out[2] == 0).all()
        _close_half(torch.from_numpy(out[1:2]), _oracle(c)[1:2], f"row 1 {kernel}")


def test_page_table_validation_messages(cuda):
    c = _random_case(3, [150, 70], 8, 8, 64, torch.float16)
    pt = torch.from_numpy(c["pt"]).clone()
    bad = pt.clone()
    bad[0, 1] = 10_000
    with pytest.raises(RuntimeError, match=r"page_table\[0\]\[1\]=10000 out of range"):
        _run(dict(c, pt=bad.numpy()))
    bad = pt.clone()
    bad[1, 2] = 0
    with pytest.raises(RuntimeError, match="must be PAD_ID"):
        _run(dict(c, pt=bad.numpy()))
    with pytest.raises(RuntimeError, match="block dim"):
        _run(dict(c, k=c["k"][:, :, :32]))
    with pytest.raises(RuntimeError, match="rope tables must cover"):
        _run(dict(c, cos=c["cos"][:64], sin=c["sin"][:64]))


def test_unchecked_bad_entry_sets_status_without_fault(cuda):
    """With validation off, the kernel's own bounds check skips the entry and reports it."""
    c = _random_case(4, [150, 70], 8, 8, 128, torch.bfloat16)
    bad = c["pt"].copy()
    bad[0, 1] = 1 << 20
    for kernel in ("tc", "simt"):
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        _run(dict(c, pt=bad), validate=False, status=status, kernel=kernel)
        torch.cuda.synchronize()
        assert int(status.item()) & 1, kernel
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    _run(c, status=status)
    assert int(status.item()) == 0


def test_long_context_checksum_property(cuda):
    """Config-3-scale lengths: attention output rows are convex combinations of V.

    With V set to a constant per KV head, every output row equals that constant
    exactly (softmax weights sum to one), whatever the scores: a size-independent
    check of the split-K combine at 30k-token contexts.
    """
    lens = [30000, 8192, 17001]
    pool = sum(-(-n // 64) for n in lens) + 3
    bt = BlockTable(pool)
    heads = [bt.allocate_chain(-(-n // 64)) for n in lens]
    pt = torch.from_numpy(build_page_table_array(bt, heads)).cuda()
    g = torch.Generator(device="cuda").manual_seed(0)
    k = (torch.randn(pool, 8, 64, 128, generator=g, device="cuda") * 0.5).to(torch.bfloat16)
    consts = torch.arange(1, 9, device="cuda", dtype=torch.float32) / 8
    v = consts.view(1, 8, 1, 1).expand(pool, 8, 64, 128).to(torch.bfloat16).contiguous()
    q = (torch.randn(3, 64, 128, generator=g, device="cuda") * 0.5).to(torch.bfloat16)
    cos, sin = ao.rope_tables(pt.shape[1] * 64, 128, 500000.0)
    out = ba.block_attention_decode(pt, q, k, v, torch.tensor(lens).cuda(),
                                    torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda())
    want = consts.repeat_interleave(8).view(1, 64, 1).expand(3, 64, 128)
    assert (out.float() - want).abs().max().item() < 1e-2


def test_tc_pipeline_under_load_reports_clean_status(cuda):
    """Many CTAs streaming long chains at once: every bounded wait must succeed.

    The status word collects the kernels' error bits (a wait that gave up sets
    bit 2); a clean run leaves it 0, and the rows still match the oracle.
    """
    rng = random.Random(8)
    lens = [rng.randint(4000, 9000) for _ in range(48)]
    pool = sum(-(-n // 64) for n in lens) + 11
    bt = BlockTable(pool)
    ids = [bt.allocate_block() for _ in range(pool)]
    rng.shuffle(ids)
    for i in ids:
        bt.free_block(i)
    heads = [bt.allocate_chain(-(-n // 64)) for n in lens]
    pt = build_page_table_array(bt, heads)
    g = torch.Generator(device="cuda").manual_seed(8)
    k = (torch.randn(pool, 8, 64, 128, generator=g, device="cuda") * 0.5).bfloat16()
    v = (torch.randn(pool, 8, 64, 128, generator=g, device="cuda") * 0.5).bfloat16()
    q = (torch.randn(len(lens), 64, 128, generator=g, device="cuda") * 0.5).bfloat16()
    cos, sin = ao.rope_tables(pt.shape[1] * 64, 128, 500000.0)
    for split in (0, 8, 24):
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        out = ba.block_attention_decode(torch.from_numpy(pt).cuda(), q, k, v,
                                        torch.tensor(lens).cuda(), torch.from_numpy(cos).cuda(),
                                        torch.from_numpy(sin).cuda(), kernel="tc",
                                        split_blocks=split, status=status)
        torch.cuda.synchronize()
        assert int(status.item()) == 0, split
        for s in (0, 17, 47):
            row = pt[s:s + 1]
            used = sorted({int(x) for x in row.reshape(-1) if x >= 0})
            remap = np.full(pool, -1, np.int32)
            remap[used] = np.arange(len(used))
            small = np.where(row >= 0, remap[np.maximum(row, 0)], -1).astype(np.int32)
            sel = torch.tensor(used, device="cuda")
            want = ao.decode_attention(small, q[s:s + 1].float().cpu().numpy(),
                                       k.index_select(0, sel).float().cpu().numpy(),
                                       v.index_select(0, sel).float().cpu().numpy(), [lens[s]],
                                       cos, sin)
            _close_half(out[s:s + 1], want, f"stress seq {s} split {split}")


@pytest.mark.parametrize("split_blocks", [0, 3])
def test_scope_skips_disallowed_blocks_vs_oracle(cuda, split_blocks):
    """Scopes that leave most blocks without an allowed key (long LOCAL
    segments away from the query, sparse GLOBAL tokens): the tensor-core
    kernel drops those blocks before loading them, split-K chunks can end up
    empty, and the rows still match the oracle."""
    rng = random.Random(21)
    lens = [5000, 3100, 64, 900, 7777, 130]
    pool = sum(-(-n // 64) for n in lens) + 5
    bt = BlockTable(pool)
    heads = [bt.allocate_chain(-(-n // 64)) for n in lens]
    pt = build_page_table_array(bt, heads)
    g = torch.Generator(device="cuda").manual_seed(21)
    k = (torch.randn(pool, 8, 64, 128, generator=g, device="cuda") * 0.5).to(torch.bfloat16)
    v = (torch.randn(pool, 8, 64, 128, generator=g, device="cuda") * 0.5).to(torch.bfloat16)
    q = (torch.randn(len(lens), 32, 128, generator=g, device="cuda") * 0.5).to(torch.bfloat16)
    W = -(-max(lens) // 16) * 16
    tags = np.zeros((len(lens), W), np.uint8)
    span = np.zeros((len(lens), 2), np.int32)
    for s, n in enumerate(lens):
        for j in rng.sample(range(n), max(1, n // 700)):   # a few GLOBAL tokens
            tags[s, j] = 1
        if s % 2 == 0:                                     # LOCAL query: its own segment
            span[s] = (max(0, n - rng.randint(1, 300)), n)
        else:                                              # GLOBAL query: itself GLOBAL
            tags[s, n - 1] = 1
    cos, sin = ao.rope_tables(pt.shape[1] * 64, 128, 500000.0)
    out = ba.block_attention_decode(torch.from_numpy(pt).cuda(), q, k, v,
                                    torch.tensor(lens).cuda(), torch.from_numpy(cos).cuda(),
                                    torch.from_numpy(sin).cuda(),
                                    scope=(torch.from_numpy(tags), torch.from_numpy(span)),
                                    kernel="tc", split_blocks=split_blocks)
    want = ao.decode_attention(pt, q.float().cpu().numpy(), k.float().cpu().numpy(),
                               v.float().cpu().numpy(), lens, cos, sin, scope_tags=tags,
                               scope_span=span)
    err = np.abs(out.float().cpu().numpy() - want)
    assert err.max() <= 2e-2 and err.mean() <= 2e-3, (err.max(), err.mean())


@pytest.mark.parametrize("kernel", ["tc", "simt"])
def test_sequence_longer_than_its_row_is_clamped_and_reported(cuda, kernel):
    """A length above 64 * max_blocks (unchecked call) reads no entry past the row:
    the kernels take the row's keys only and set status bit 1; a max_seq_blocks bound
    below a sequence's blocks does the same at that bound."""
    c = _random_case(31, [1000, 300, 640], 16, 2, 128, torch.bfloat16)
    max_b = c["pt"].shape[1]                       # 16 blocks: sequence 0's full row
    long = c["lens"].copy()
    long[0] = 64 * max_b + 1                       # one key past the row
    pos = np.asarray([999, 299, 639], np.int32)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = _run(dict(c, lens=long), validate=False, status=status, kernel=kernel,
               positions=torch.from_numpy(pos).cuda(), split_blocks=3)
    torch.cuda.synchronize()
    assert int(status.item()) & 1
    clamped = long.copy()
    clamped[0] = 64 * max_b
    _close_half(out, _oracle(dict(c, lens=clamped), positions=pos), f"row clamp {kernel}")
    # the host bound: no sequence past 10 blocks (sequence 0 has 16)
    status.zero_()
    out = _run(c, validate=False, status=status, kernel=kernel, max_seq_blocks=10,
               total_blocks=10 + 5 + 10)
    torch.cuda.synchronize()
    assert int(status.item()) & 1
    capped = np.minimum(c["lens"], 640)
    _close_half(out, _oracle(dict(c, lens=capped), positions=c["lens"] - 1), f"cap {kernel}")


def test_total_blocks_hint_plans_from_the_real_work(cuda):
    """A wide table holding short chains: with total_blocks the planner sizes the
    chunks from the batch's blocks, not from the width; the rows still match."""
    rng = random.Random(41)
    lens = [rng.randint(64, 900) for _ in range(200)] + [30000]
    c = _random_case(41, lens, 64, 8, 128, torch.bfloat16)
    args = [torch.from_numpy(c[x]).cuda() if isinstance(c[x], np.ndarray) else c[x].cuda()
            for x in ("pt", "q", "k", "v", "lens", "cos", "sin")]
    blind = ba.DecodeCall(*args, kernel="tc")
    total = int(sum(-(-n // 64) for n in lens))
    aware = ba.DecodeCall(*args, total_blocks=total, max_seq_blocks=c["pt"].shape[1],
                          kernel="tc")
    assert aware.plan["split_blocks"] < blind.plan["split_blocks"]
    _close_half(aware.launch(), _oracle(c), "planned from total_blocks")
