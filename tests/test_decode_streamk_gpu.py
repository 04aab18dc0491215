"""Stream-K tensor-core decode (kernel="streamk") on the GPU vs the oracle.

One persistent CTA per SM takes an equal share of the batch's blocks, sequence
after sequence; every consumer warp writes its state per sequence piece and a
merge kernel combines the pieces. These tests cover the piece bookkeeping:
sequences spread over many CTAs and CTAs spanning many sequences, empty and
one-token sequences, shares longer than one window of the block list (forced
with a small CTA count), more sequences in a share than one window holds, GQA
groups 1-8, head_dim 64 and 128, the token scope and block mask, and a clean
status word. Tolerance: the fp16/bf16 bar (max-abs 2e-2, mean-abs 2e-3).
"""

import random

import numpy as np
import pytest
import torch

from oracle import attention_oracle as ao
from src.block_table import BlockTable, build_page_table_array
from src.kernels import block_attention as ba

pytestmark = pytest.mark.gpu
HALF_MAX, HALF_MEAN = 2e-2, 2e-3


def _case(lens, hq, hkv, d, dtype, seed):
    rng = random.Random(seed)
    pool = sum(max(1, -(-n // 64)) for n in lens) + 7
    bt = BlockTable(pool)
    ids = [bt.allocate_block() for _ in range(pool)]
    rng.shuffle(ids)
    for i in ids:
        bt.free_block(i)
    heads = [bt.allocate_chain(max(1, -(-n // 64))) for n in lens]
    pt = build_page_table_array(bt, heads)
    for s, n in enumerate(lens):
        pt[s, -(-n // 64):] = -1  # an empty sequence's row holds no block
    g = torch.Generator(device="cuda").manual_seed(seed)
    k = (torch.randn(pool, hkv, 64, d, generator=g, device="cuda") * 0.5).to(dtype)
    v = (torch.randn(pool, hkv, 64, d, generator=g, device="cuda") * 0.5).to(dtype)
    q = (torch.randn(len(lens), hq, d, generator=g, device="cuda") * 0.5).to(dtype)
    cos, sin = ao.rope_tables(pt.shape[1] * 64, d, 500000.0)
    return dict(pt=pt, q=q, k=k, v=v, lens=np.asarray(lens, np.int32), cos=cos, sin=sin)


def _run(c, **kw):
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = ba.block_attention_decode(torch.from_numpy(c["pt"]).cuda(), c["q"], c["k"], c["v"],
                                    torch.from_numpy(c["lens"]).cuda(),
                                    torch.from_numpy(c["cos"]).cuda(),
                                    torch.from_numpy(c["sin"]).cuda(), kernel="streamk",
                                    status=status, **kw)
    torch.cuda.synchronize()
    assert int(status.item()) == 0, int(status.item())
    return out


def _check(c, out, rows=None, **okw):
    rows = list(range(len(c["lens"]))) if rows is None else rows
    pt = c["pt"][rows]
    used = sorted({int(x) for x in pt.reshape(-1) if x >= 0})
    remap = np.full(c["k"].shape[0], -1, np.int32)
    remap[used] = np.arange(len(used))
    small = np.where(pt >= 0, remap[np.maximum(pt, 0)], -1).astype(np.int32)
    sel = torch.tensor(used, device="cuda")
    kw = {k: (v[rows] if isinstance(v, np.ndarray) else v) for k, v in okw.items()}
    want = ao.decode_attention(small, c["q"][rows].float().cpu().numpy(),
                               c["k"].index_select(0, sel).float().cpu().numpy(),
                               c["v"].index_select(0, sel).float().cpu().numpy(),
                               c["lens"][rows], c["cos"], c["sin"], **kw)
    err = np.abs(out[rows].float().cpu().numpy() - want)
    assert err.max() <= HALF_MAX and err.mean() <= HALF_MEAN, (err.max(), err.mean())


@pytest.mark.parametrize("hq,hkv,d,dtype", [(64, 8, 128, torch.bfloat16),
                                            (32, 8, 128, torch.float16),
                                            (8, 8, 64, torch.float16),
                                            (12, 2, 128, torch.bfloat16),
                                            (5, 1, 64, torch.bfloat16)])
def test_streamk_ragged_batch_vs_oracle(cuda, hq, hkv, d, dtype):
    rng = random.Random(hq * 7 + hkv)
    lens = [rng.randint(1, 9000) for _ in range(40)] + [0, 1, 64, 65, 30000]
    c = _case(lens, hq, hkv, d, dtype, seed=hq + d)
    _check(c, _run(c))


@pytest.mark.parametrize("ctas", [1, 2, 3, 7])
def test_streamk_shares_longer_than_one_window(cuda, ctas):
    """A few CTAs per KV-head group: each share spans windows of the block list and
    cuts sequences at window boundaries (state carried in registers)."""
    lens = [20000, 7000, 13, 4096, 9999, 64 * 768 + 5, 1]
    c = _case(lens, 64, 8, 128, torch.bfloat16, seed=ctas)
    _check(c, _run(c, split_blocks=ctas))


def test_streamk_many_sequences_per_share(cuda):
    """Thousands of one- and two-block sequences: every CTA's share holds more
    sequences than one window lists."""
    rng = random.Random(5)
    lens = [rng.randint(1, 128) for _ in range(6000)]
    c = _case(lens, 32, 8, 128, torch.bfloat16, seed=5)
    out = _run(c)
    _check(c, out, rows=list(range(0, 6000, 97)) + [5999])


def test_streamk_scope_and_block_mask(cuda):
    rng = random.Random(21)
    lens = [5000, 3100, 64, 900, 7777, 130, 0]
    c = _case(lens, 32, 8, 128, torch.bfloat16, seed=21)
    W = -(-max(lens) // 16) * 16
    tags = np.zeros((len(lens), W), np.uint8)
    span = np.zeros((len(lens), 2), np.int32)
    for s, n in enumerate(lens):
        if n == 0:
            continue
        for j in rng.sample(range(n), max(1, n // 700)):
            tags[s, j] = 1
        span[s] = (max(0, n - rng.randint(1, 300)), n)
    out = _run(c, scope=(torch.from_numpy(tags), torch.from_numpy(span)))
    _check(c, out, scope_tags=tags, scope_span=span)
    nb = c["pt"].shape[1]
    mask = (np.random.default_rng(3).random((len(lens), nb, nb)) < 0.5).astype(np.int8)
    out = _run(c, mask=torch.from_numpy(mask), split_blocks=5)
    _check(c, out, block_mask=mask)


def test_streamk_matches_split_k_on_the_workload_shape(cuda):
    """The 70B-shape batch (GQA 64/8, lens U[8192, 32768]) on 32 sequences: stream-K
    and split-K agree with each other and with the oracle on a few rows."""
    rng = random.Random(1234)
    lens = [rng.randint(8192, 32768) for _ in range(32)]
    c = _case(lens, 64, 8, 128, torch.bfloat16, seed=3)
    out = _run(c)
    ref = ba.block_attention_decode(torch.from_numpy(c["pt"]).cuda(), c["q"], c["k"], c["v"],
                                    torch.from_numpy(c["lens"]).cuda(),
                                    torch.from_numpy(c["cos"]).cuda(),
                                    torch.from_numpy(c["sin"]).cuda(), kernel="tc")
    err = (out.float() - ref.float()).abs()
    assert err.max().item() <= HALF_MAX and err.mean().item() <= HALF_MEAN
    _check(c, out, rows=[0, 17, 31])


@pytest.mark.parametrize("hq,hkv,d,dtype", [(32, 8, 128, torch.float16),
                                            (3, 1, 64, torch.bfloat16)])
def test_streamk_fewer_blocks_than_ctas(cuda, hq, hkv, d, dtype):
    """A batch of 76 blocks over 148 CTAs: CTAs between a sequence's first and last own
    no block; the merge skips their slots."""
    lens = [1, 63, 64, 65, 700, 2049, 1500, 129]
    c = _case(lens, hq, hkv, d, dtype, seed=hq * 7 + d)
    _check(c, _run(c))
    _check(c, _run(c, split_blocks=100))
