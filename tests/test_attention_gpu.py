"""The reference's block_attention entry (full self-attention) and chunked prefill on the GPU.

The fp32 / fp16 cases replay the reference's own GPU tests'
shapes (tests/test_block_attention.py:278-360): 2 sequences x 3 blocks, H=2,
D=32, with and without additive bias + block mask, against the outputs the
reference's dense_reference recorded (tests/golden/attn_small.npz), plus the
reference's validation messages.
"""

from pathlib import Path

import numpy as np
import pytest
import torch

import cases
from oracle import attention_oracle as ao
from src.block_table import BlockTable, build_page_table_array
from src.kernels import block_attention as ba

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"


def _case(name):
    seed = {"bm": 1234, "plain": 77, "f16": 5}[name]
    dt = torch.float16 if name == "f16" else torch.float32
    c = cases.small_full_case(torch, BlockTable, seed, dtype=dt)
    kw = {}
    if name == "bm":
        gen = torch.Generator().manual_seed(seed + 1)
        bias = torch.randn(1, 2, max(c["lens"]), max(c["lens"]), generator=gen) * 0.25
        scope = torch.randint(0, 2, (2, 3, 3), generator=gen) | torch.eye(3, dtype=torch.int64)
        kw = dict(bias=bias.cuda(), mask=scope.to(torch.int8).cuda())
    return c, kw


@pytest.mark.parametrize("name,tol", [("bm", 2e-3), ("plain", 2e-3), ("f16", 2e-2)])
def test_block_attention_matches_reference(cuda, name, tol):
    g = np.load(GOLD / "attn_small.npz")
    c, kw = _case(name)
    pt = torch.tensor(c["rows"], dtype=torch.int32).cuda()
    out = ba.block_attention(pt, c["q_cache"].cuda(), c["k_cache"].cuda(), c["v_cache"].cuda(),
                             torch.tensor(c["lens"], dtype=torch.int32).cuda(), c["cos"].cuda(),
                             c["sin"].cuda(), **kw)
    assert out.shape == g[f"{name}_out"].shape and out.dtype == c["q_cache"].dtype
    err = np.abs(out.float().cpu().numpy() - g[f"{name}_out"])
    assert err.max() < tol, err.max()


def test_block_attention_cpu_inputs_are_moved(cuda):
    c, _ = _case("plain")
    out = ba.block_attention(torch.tensor(c["rows"]), c["q_cache"], c["k_cache"].cuda(),
                             c["v_cache"], torch.tensor(c["lens"]), c["cos"], c["sin"])
    assert out.is_cuda


def test_block_attention_validates_before_launch(cuda):
    c, _ = _case("plain")
    pt = torch.tensor(c["rows"], dtype=torch.int32).cuda()
    args = [c["q_cache"].cuda(), c["k_cache"].cuda(), c["v_cache"].cuda(),
            torch.tensor(c["lens"]).cuda(), c["cos"].cuda(), c["sin"].cuda()]
    bad = pt.clone()
    bad[0, 0] = 999
    with pytest.raises(RuntimeError, match="out of range"):
        ba.block_attention(bad, *args)
    with pytest.raises(RuntimeError, match="block dim"):
        ba.block_attention(pt, args[0][:, :, :32, :], *args[1:])
    small = [t[..., :8].contiguous() for t in args[:3]]
    cos8, sin8 = ao.rope_tables(pt.shape[1] * 64, 8)
    with pytest.raises(RuntimeError, match="head dim"):
        ba.block_attention(pt, *small, args[3], torch.from_numpy(cos8), torch.from_numpy(sin8))


@pytest.mark.parametrize("hq,hkv,dtype", [(8, 2, torch.bfloat16), (4, 4, torch.float32)])
def test_chunked_prefill_vs_oracle(cuda, hq, hkv, dtype):
    lens_total = [700, 300, 1024]
    starts = [512, 200, 512]
    L = 512
    bt = BlockTable(64)
    heads = [bt.allocate_chain(-(-n // 64)) for n in lens_total]
    pt = build_page_table_array(bt, heads)
    g = torch.Generator().manual_seed(3)
    k = (torch.randn(64, hkv, 64, 64, generator=g) * 0.5).to(dtype)
    v = (torch.randn(64, hkv, 64, 64, generator=g) * 0.5).to(dtype)
    q = (torch.randn(3, hq, L, 64, generator=g) * 0.5).to(dtype)
    cos, sin = ao.rope_tables(pt.shape[1] * 64, 64, 500000.0)
    out = ba.chunked_prefill_attention(torch.from_numpy(pt).cuda(), q.cuda(), k.cuda(), v.cuda(),
                                       torch.tensor(starts).cuda(), torch.tensor(lens_total).cuda(),
                                       torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda())
    want = ao.prefill_attention(pt, q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                starts, lens_total, cos, sin, causal=True)
    err = np.abs(out.float().cpu().numpy() - want)
    tol = 2e-2 if dtype != torch.float32 else 1e-4
    assert err.max() < tol and err.mean() < 2e-3, (err.max(), err.mean())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("with_mask", [False, True])
def test_block_attention_on_tensor_cores_vs_oracle(cuda, dtype, with_mask):
    """The drop-in full self-attention on the tcgen05 kernel (paged queries, D 128):
    ragged lengths (one block, a partial last block, several 128-row query tiles),
    optionally a block mask with the diagonal kept; every valid row vs the oracle and
    vs the CUDA-core kernel."""
    lens = [700, 1100, 64, 200, 129]
    H, D = 8, 128
    bt, heads, rows = cases.scattered_chains(BlockTable, 64, lens, 33)
    q, k, v = cases.paged_caches(torch, 33, 64, H, D, 0.5, dtype)
    cos, sin = cases.rope_tables_torch(torch, len(rows[0]) * 64, D, 10000.0)
    pt = torch.tensor(rows, dtype=torch.int32)
    kw = {}
    if with_mask:
        qb = -(-max(lens) // 64)
        gen = torch.Generator().manual_seed(9)
        m = (torch.rand(len(lens), qb, qb, generator=gen) < 0.6).to(torch.int8)
        m |= torch.eye(qb, dtype=torch.int8)
        kw = dict(mask=m)
    args = (pt.cuda(), q.cuda(), k.cuda(), v.cuda(), torch.tensor(lens).cuda(), cos.cuda(),
            sin.cuda())
    got = ba.block_attention(*args, kernel="tc", **{k2: x.cuda() for k2, x in kw.items()})
    simt = ba.block_attention(*args, kernel="simt", **{k2: x.cuda() for k2, x in kw.items()})
    want = ao.dense_attention(pt.numpy(), q.float().numpy(), k.float().numpy(),
                              v.float().numpy(), lens, cos.numpy(), sin.numpy(),
                              mask=kw["mask"].numpy() if with_mask else None)
    for out in (got, simt):
        errs = np.concatenate([np.abs(out[s, :, :n].float().cpu().numpy() - want[s, :, :n])
                               .reshape(-1) for s, n in enumerate(lens)])
        assert errs.max() <= 2e-2 and errs.mean() <= 2e-3, (errs.max(), errs.mean())
    # rows past each sequence stay zero
    for s, n in enumerate(lens):
        assert got[s, :, n:].abs().max().item() == 0 if n < max(lens) else True


def test_block_attention_auto_picks_tensor_cores_without_bias(cuda):
    """kernel='auto' takes the tensor-core kernel for fp16/bf16, D 128, no bias, and the
    CUDA-core kernel with an additive bias; both agree with the oracle."""
    lens = [300, 513]
    H, D = 4, 128
    bt, heads, rows = cases.scattered_chains(BlockTable, 32, lens, 7)
    q, k, v = cases.paged_caches(torch, 7, 32, H, D, 0.5, torch.bfloat16)
    cos, sin = cases.rope_tables_torch(torch, len(rows[0]) * 64, D, 10000.0)
    pt = torch.tensor(rows, dtype=torch.int32)
    bias = torch.randn(1, H, max(lens), max(lens), generator=torch.Generator().manual_seed(1))
    for kw in ({}, dict(bias=bias * 0.25)):
        out = ba.block_attention(pt.cuda(), q.cuda(), k.cuda(), v.cuda(),
                                 torch.tensor(lens).cuda(), cos.cuda(), sin.cuda(),
                                 **{k2: x.cuda() for k2, x in kw.items()})
        want = ao.dense_attention(pt.numpy(), q.float().numpy(), k.float().numpy(),
                                  v.float().numpy(), lens, cos.numpy(), sin.numpy(),
                                  bias=kw["bias"].numpy() if kw else None)
        for s, n in enumerate(lens):
            e = np.abs(out[s, :, :n].float().cpu().numpy() - want[s, :, :n])
            assert e.max() <= 2e-2 and e.mean() <= 2e-3, (kw.keys(), e.max(), e.mean())
