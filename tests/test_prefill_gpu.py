"""Chunked prefill on the tcgen05 tensor-core kernel vs the oracle.

Tolerance: max-abs 2e-2 and mean-abs 2e-3 (fp16/bf16) against the fp32
oracle's prefill rows (the row form of dense_reference with a causal bias).
Every launch also passes a status word that must stay 0 (no bounded wait
gave up, no bad page entry).
"""

import random

import numpy as np
import pytest
import torch

from oracle import attention_oracle as ao
from src.block_table import BlockTable, build_page_table_array
from src.kernels import block_attention as ba

pytestmark = pytest.mark.gpu


def _case(seed, totals, hq, hkv, L, dtype, d=128, base=500000.0):
    rng = random.Random(seed)
    pool = sum(-(-n // 64) for n in totals) + 9
    bt = BlockTable(pool)
    ids = [bt.allocate_block() for _ in range(pool)]
    rng.shuffle(ids)
    for i in ids:
        bt.free_block(i)
    heads = [bt.allocate_chain(-(-n // 64)) for n in totals]
    pt = build_page_table_array(bt, heads)
    g = torch.Generator(device="cuda").manual_seed(seed)
    k = (torch.randn(pool, hkv, 64, d, generator=g, device="cuda") * 0.5).to(dtype)
    v = (torch.randn(pool, hkv, 64, d, generator=g, device="cuda") * 0.5).to(dtype)
    q = (torch.randn(len(totals), hq, L, d, generator=g, device="cuda") * 0.5).to(dtype)
    cos, sin = ao.rope_tables(pt.shape[1] * 64, d, base)
    return pt, q, k, v, cos, sin


def _run(pt, q, k, v, starts, totals, cos, sin, **kw):
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = ba.chunked_prefill_attention(torch.from_numpy(pt).cuda(), q, k, v,
                                       torch.tensor(starts).cuda(), torch.tensor(totals).cuda(),
                                       torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda(),
                                       status=status, **kw)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return out


def _check(out, want, label):
    err = np.abs(out.float().cpu().numpy() - want)
    assert err.max() <= 2e-2 and err.mean() <= 2e-3, (label, err.max(), err.mean())


@pytest.mark.parametrize("hq,hkv,dtype,causal", [
    (32, 8, torch.bfloat16, True),     # Llama-3-8B attention shape (group 4)
    (4, 4, torch.bfloat16, False),     # MHA, non-causal
    (16, 2, torch.float16, True),      # group 8
    (8, 4, torch.bfloat16, True),      # group 2
])
def test_tensor_core_prefill_vs_oracle(cuda, hq, hkv, dtype, causal):
    L = 512
    starts = [512, 0, 1024]
    totals = [1024, 300, 1100]          # second and third sequences end inside the chunk
    pt, q, k, v, cos, sin = _case(hq + hkv, totals, hq, hkv, L, dtype)
    out = _run(pt, q, k, v, starts, totals, cos, sin, causal=causal, kernel="tc")
    want = ao.prefill_attention(pt, q.float().cpu().numpy(), k.float().cpu().numpy(),
                                v.float().cpu().numpy(), starts, totals, cos, sin, causal=causal)
    _check(out, want, f"{hq}/{hkv} causal={causal}")
    # rows past the sequence end are left untouched (zero-initialised output)
    assert (out[1, :, 300:].float() == 0).all()


@pytest.mark.parametrize("hq,hkv,causal", [(32, 8, True), (16, 16, True), (32, 4, False)])
def test_persistent_ctas_many_ragged_items(cuda, hq, hkv, causal):
    """More work items than SMs, so each CTA walks several items back to back:
    one-tile items, odd tile counts (the S/P buffer parity flips between
    items), rows past the sequence end and chunks that start mid-sequence."""
    rng = random.Random(hq * 7 + hkv + causal)
    L = 256
    totals = [rng.randint(1, 1700) for _ in range(7)] + [37, 300]
    starts = [max(0, t - rng.randint(1, L + 64)) for t in totals]
    pt, q, k, v, cos, sin = _case(100 + hq + hkv, totals, hq, hkv, L, torch.bfloat16)
    out = _run(pt, q, k, v, starts, totals, cos, sin, causal=causal, kernel="tc")
    want = ao.prefill_attention(pt, q.float().cpu().numpy(), k.float().cpu().numpy(),
                                v.float().cpu().numpy(), starts, totals, cos, sin, causal=causal)
    rows = [min(L, t - s) for s, t in zip(starts, totals)]
    for i, n in enumerate(rows):     # only rows inside the sequence are written
        _check(out[i:i + 1, :, :n], want[i:i + 1, :, :n], f"seq {i} ({starts[i]}+{n}/{totals[i]})")
        assert (out[i, :, n:].float() == 0).all()


@pytest.mark.parametrize("hq,hkv,L", [(32, 2, 100), (64, 2, 37), (128, 1, 9)])
def test_large_gqa_groups_few_positions_per_item(cuda, hq, hkv, L):
    """Groups of 16, 32 and 128 query heads: 8, 4 and 1 positions per 128-row
    item, chunk lengths that leave the last item partly empty."""
    starts, totals = [300, 0, 1000], [400, 20, 1009]
    pt, q, k, v, cos, sin = _case(hq * 3 + L, totals, hq, hkv, L, torch.bfloat16)
    out = _run(pt, q, k, v, starts, totals, cos, sin, causal=True, kernel="tc")
    want = ao.prefill_attention(pt, q.float().cpu().numpy(), k.float().cpu().numpy(),
                                v.float().cpu().numpy(), starts, totals, cos, sin, causal=True)
    _check(out, want, f"{hq}/{hkv} L={L}")


def test_chunked_prefill_reuses_rotated_keys(cuda):
    """One workspace across the chunks of a prefill with krot_valid = tokens
    already rotated. After each chunk the K cache rows of those tokens are
    overwritten with garbage: later chunks still match the oracle on the
    original keys, so the rotated scratch (not the cache) serves them."""
    hq, hkv, d, L, chunks = 32, 8, 128, 256, 4
    totals = [L * chunks] * 3
    pt, q_all, k, v, cos, sin = _case(55, totals, hq, hkv, L * chunks, torch.bfloat16)
    k_orig = k.clone()
    want = ao.prefill_attention(pt, q_all.float().cpu().numpy(), k_orig.float().cpu().numpy(),
                                v.float().cpu().numpy(), [0] * 3, totals, cos, sin, causal=True)
    ptd = torch.from_numpy(pt).cuda()
    cos_d, sin_d = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
    ws = None  # the first call allocates the workspace; the later ones reuse it
    for c in range(chunks):
        starts = torch.full((3,), c * L, dtype=torch.int32, device="cuda")
        lens = torch.full((3,), (c + 1) * L, dtype=torch.int32, device="cuda")
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        pt_c = ptd.clone()  # the chains as they stand after chunk c (PAD past them)
        pt_c[:, (c + 1) * L // 64:] = -1
        call = ba.PrefillCall(pt_c, q_all[:, :, c * L:(c + 1) * L].contiguous(), k, v, starts, lens,
                              cos_d, sin_d, kernel="tc", status=status, workspace=ws,
                              krot_valid=torch.full((3,), c * L, dtype=torch.int32))
        ws = call.workspace
        out = call.launch()
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        _check(out, want[:, :, c * L:(c + 1) * L], f"chunk {c}")
        # corrupt every key rotated so far (its blocks are not read again)
        for s in range(3):
            for b in range((c + 1) * L // 64):
                k[pt[s, b]] = 7.0


def test_key_rotation_many_units_per_cta(cuda):
    """A 32-token chunk at the end of ~9k-token sequences: 16 work items, so 16
    CTAs rotate 564 units of 64 keys x 4 KV heads (several lookup batches per
    CTA). A second launch on the same workspace with krot_valid inside a block
    (100, 4000) re-rotates only from that block on: the cache rows of the
    blocks wholly below it are overwritten first and must not matter."""
    hq, hkv, L = 32, 8, 32
    totals = [9000, 8500]
    starts = [t - L for t in totals]
    pt, q, k, v, cos, sin = _case(77, totals, hq, hkv, L, torch.bfloat16)
    want = ao.prefill_attention(pt, q.float().cpu().numpy(), k.float().cpu().numpy(),
                                v.float().cpu().numpy(), starts, totals, cos, sin, causal=True)
    ptd = torch.from_numpy(pt).cuda()
    cos_d, sin_d = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
    starts_d = torch.tensor(starts, dtype=torch.int32, device="cuda")
    lens_d = torch.tensor(totals, dtype=torch.int32, device="cuda")
    ws = None
    for kv in (None, [100, 4000]):
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        call = ba.PrefillCall(ptd, q, k, v, starts_d, lens_d, cos_d, sin_d, kernel="tc",
                              status=status, workspace=ws,
                              krot_valid=None if kv is None else torch.tensor(kv, dtype=torch.int32))
        ws = call.workspace
        out = call.launch()
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        _check(out, want, f"krot_valid={kv}")
        if kv is None:
            for s_, kv_s in enumerate([100, 4000]):
                for b in range(kv_s // 64):
                    k[pt[s_, b]] = 7.0


@pytest.mark.parametrize("hq,hkv,dtype,kernel", [
    (32, 8, torch.bfloat16, "tc"), (16, 2, torch.float16, "tc"), (8, 4, torch.float32, "simt")])
def test_prefill_with_token_scope_vs_oracle(cuda, hq, hkv, dtype, kernel):
    """Table-1 token scope (GLOBAL tags + each query position's LOCAL span) on
    top of causality, chunks starting mid-sequence, ragged lengths."""
    from src.scoping_mask import prefill_scope
    from src.engine import random_segments

    rng = random.Random(hq + hkv)
    L = 384
    totals = [1000, 400, 777, 1300]
    starts = [600, 0, 700, 1000]
    spans = [random_segments(rng, t) for t in totals]
    tags, lo, hi = prefill_scope(spans)
    d = 128 if kernel == "tc" else 64
    pt, q, k, v, cos, sin = _case(77 + hq, totals, hq, hkv, L, dtype, d=d)
    out = _run(pt, q, k, v, starts, totals, cos, sin, causal=True, kernel=kernel,
               scope=(torch.from_numpy(tags), torch.from_numpy(lo), torch.from_numpy(hi)))
    want = ao.prefill_attention(pt, q.float().cpu().numpy(), k.float().cpu().numpy(),
                                v.float().cpu().numpy(), starts, totals, cos, sin, causal=True,
                                scope_tags=tags, scope_lo=lo, scope_hi=hi)
    tol = (2e-2, 2e-3) if dtype != torch.float32 else (1e-4, 1e-5)
    err = np.abs(out.float().cpu().numpy() - want)
    assert err.max() <= tol[0] and err.mean() <= tol[1], (err.max(), err.mean())


def test_tensor_cores_agree_with_cuda_cores(cuda):
    L, starts, totals = 256, [64, 700], [320, 956]
    pt, q, k, v, cos, sin = _case(7, totals, 32, 8, L, torch.bfloat16)
    a = _run(pt, q, k, v, starts, totals, cos, sin, kernel="tc")
    b = _run(pt, q, k, v, starts, totals, cos, sin, kernel="simt")
    _check(a, b.float().cpu().numpy(), "tc vs simt")


def test_two_chunk_prefill_through_kv_append(cuda):
    """Config-4 flow at small scale: each 512-token chunk's K/V is appended into
    newly allocated blocks, then the chunk attends to everything before it."""
    hq, hkv, d, L, chunks, S = 32, 8, 128, 512, 2, 2
    total = L * chunks
    bt = BlockTable(64)
    heads = [bt.allocate_chain(L // 64) for _ in range(S)]
    g = torch.Generator(device="cuda").manual_seed(3)
    kc = torch.zeros(64, hkv, 64, d, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    cos, sin = ao.rope_tables(total, d, 500000.0)
    q_all = (torch.randn(S, hq, total, d, generator=g, device="cuda") * 0.5).bfloat16()
    k_all = (torch.randn(S, hkv, total, d, generator=g, device="cuda") * 0.5).bfloat16()
    v_all = (torch.randn(S, hkv, total, d, generator=g, device="cuda") * 0.5).bfloat16()
    outs = []
    for c in range(chunks):
        if c > 0:                                   # [EXPAND]: grow each chain by one chunk
            for h in heads:
                tail = bt.chain_tail(h)
                for _ in range(L // 64):
                    tail = bt.expand_chain(tail)
        pt = torch.from_numpy(build_page_table_array(bt, heads, pad_to=total // 64)).cuda()
        start = torch.full((S,), c * L, dtype=torch.int32, device="cuda")
        cnt = torch.full((S,), L, dtype=torch.int32, device="cuda")
        ba.paged_kv_append(k_all[:, :, c * L:(c + 1) * L], v_all[:, :, c * L:(c + 1) * L], pt,
                           start, cnt, kc, vc)
        lens = torch.full((S,), (c + 1) * L, dtype=torch.int32, device="cuda")
        outs.append(ba.chunked_prefill_attention(pt, q_all[:, :, c * L:(c + 1) * L], kc, vc,
                                                 start, lens, torch.from_numpy(cos).cuda(),
                                                 torch.from_numpy(sin).cuda(), kernel="tc"))
    got = torch.cat(outs, dim=2).float().cpu().numpy()
    # oracle: one dense causal pass over the whole prompt
    pt_final = build_page_table_array(bt, heads, pad_to=total // 64)
    want = ao.prefill_attention(pt_final, q_all.float().cpu().numpy(), kc.float().cpu().numpy(),
                                vc.float().cpu().numpy(), [0] * S, [total] * S, cos, sin,
                                causal=True)
    err = np.abs(got - want)
    assert err.max() <= 2e-2 and err.mean() <= 2e-3, (err.max(), err.mean())


@pytest.mark.parametrize("chunks", [2, 6])
def test_chained_chunk_launches_vs_oracle(cuda, chunks):
    """The chunks of a prefill launched back to back as one chain (launch_seq = chunk):
    each launch may start during the previous one's tail; it reads the previous launch's
    keys once that launch's rotation counter is complete and earlier keys at once. Two
    passes of the chain in a row: the second starts a new chain on the same workspace."""
    hq, hkv, d, L = 32, 8, 128, 256
    totals = [L * chunks] * 4
    pt, q_all, k, v, cos, sin = _case(77, totals, hq, hkv, L * chunks, torch.bfloat16)
    want = ao.prefill_attention(pt, q_all.float().cpu().numpy(), k.float().cpu().numpy(),
                                v.float().cpu().numpy(), [0] * 4, totals, cos, sin, causal=True)
    ptd = torch.from_numpy(pt).cuda()
    cos_d, sin_d = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    calls, ws = [], None
    for c in range(chunks):
        starts = torch.full((4,), c * L, dtype=torch.int32, device="cuda")
        lens = torch.full((4,), (c + 1) * L, dtype=torch.int32, device="cuda")
        pt_c = ptd.clone()
        pt_c[:, (c + 1) * L // 64:] = -1
        calls.append(ba.PrefillCall(pt_c, q_all[:, :, c * L:(c + 1) * L].contiguous(), k, v,
                                    starts, lens, cos_d, sin_d, kernel="tc", status=status,
                                    workspace=ws,
                                    krot_valid=torch.full((4,), c * L, dtype=torch.int32),
                                    launch_seq=c))
        ws = calls[-1].workspace
    for _ in range(2):
        results = [cl.launch() for cl in calls]   # no synchronisation between the launches
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        for c in range(chunks):
            _check(results[c], want[:, :, c * L:(c + 1) * L], f"chunk {c}")


def test_chained_launches_with_kv_append_between_them(cuda):
    """Serving-style chunked prefill with nothing synchronised: before each chunk's launch
    (launch_seq = chunk, one shared workspace) a kv-append kernel writes that chunk's K/V
    into the cache. Every prefill thread waits for the previous kernel on the stream before
    it touches memory, so each launch reads the keys and values just appended."""
    hq, hkv, d, L, chunks, S = 32, 8, 128, 256, 4, 3
    total = L * chunks
    bt = BlockTable(S * total // 64 + 8)
    heads = [bt.allocate_chain(total // 64) for _ in range(S)]
    ptd = torch.from_numpy(build_page_table_array(bt, heads, pad_to=total // 64)).cuda()
    g = torch.Generator(device="cuda").manual_seed(11)
    kc = torch.zeros(S * total // 64 + 8, hkv, 64, d, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    cos, sin = ao.rope_tables(total, d, 500000.0)
    cos_d, sin_d = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
    q_all = (torch.randn(S, hq, total, d, generator=g, device="cuda") * 0.5).bfloat16()
    k_all = (torch.randn(S, hkv, total, d, generator=g, device="cuda") * 0.5).bfloat16()
    v_all = (torch.randn(S, hkv, total, d, generator=g, device="cuda") * 0.5).bfloat16()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    calls, ws = [], None
    for c in range(chunks):                     # checked and prepared before any launch
        pt_c = ptd.clone()
        pt_c[:, (c + 1) * L // 64:] = -1
        calls.append(ba.PrefillCall(
            pt_c, q_all[:, :, c * L:(c + 1) * L].contiguous(), kc, vc,
            torch.full((S,), c * L, dtype=torch.int32, device="cuda"),
            torch.full((S,), (c + 1) * L, dtype=torch.int32, device="cuda"), cos_d, sin_d,
            kernel="tc", status=status, workspace=ws,
            krot_valid=torch.full((S,), c * L, dtype=torch.int32), launch_seq=c))
        ws = calls[-1].workspace
    start = [torch.full((S,), c * L, dtype=torch.int32, device="cuda") for c in range(chunks)]
    cnt = torch.full((S,), L, dtype=torch.int32, device="cuda")
    outs = []
    for c in range(chunks):                     # append, attend, append, attend, ... unsynchronised
        ba.paged_kv_append(k_all[:, :, c * L:(c + 1) * L].contiguous(),
                           v_all[:, :, c * L:(c + 1) * L].contiguous(), ptd, start[c], cnt, kc, vc)
        outs.append(calls[c].launch())
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    pt_np = build_page_table_array(bt, heads, pad_to=total // 64)
    want = ao.prefill_attention(pt_np, q_all.float().cpu().numpy(), kc.float().cpu().numpy(),
                                vc.float().cpu().numpy(), [0] * S, [total] * S, cos, sin,
                                causal=True)
    for c in range(chunks):
        _check(outs[c], want[:, :, c * L:(c + 1) * L], f"chunk {c}")
