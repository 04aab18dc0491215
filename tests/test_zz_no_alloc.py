"""The allocation-free decode entry point (ouro_paged_decode_noalloc).

Some callers cannot allocate device memory while they run: a serving loop
their host framework is capturing into a CUDA graph, a process held to a
fixed memory budget, or an application whose allocator this library cannot
reach. For them the library keeps the split-K scratch in a fixed device array
instead of asking for a workspace. This file checks that entry point through
the C ABI against the allocating one (ouro_paged_decode), on two calls in a
row, and that an explicit split the array cannot hold is refused.

It is named to be collected last, so a failure here never hides another test.
"""

import ctypes
import random

import numpy as np
import pytest
import torch

from oracle import attention_oracle as ao
from src import _native
from src.block_table import BlockTable, build_page_table_array
from src.kernels import block_attention as ba

pytestmark = pytest.mark.gpu

HALF_MAX, HALF_MEAN = 2e-2, 2e-3   # the fp16/bf16 tolerance the other decode tests use


def _case(lens, hq, hkv, d, seed):
    rng = random.Random(seed)
    pool = sum(-(-n // 64) for n in lens) + 5
    bt = BlockTable(pool)
    ids = [bt.allocate_block() for _ in range(pool)]
    rng.shuffle(ids)
    for i in ids:
        bt.free_block(i)
    heads = [bt.allocate_chain(-(-n // 64)) for n in lens]
    pt = torch.from_numpy(build_page_table_array(bt, heads)).cuda()
    g = torch.Generator(device="cuda").manual_seed(seed)
    k = (torch.randn(pool, hkv, 64, d, generator=g, device="cuda") * 0.5).bfloat16()
    v = (torch.randn(pool, hkv, 64, d, generator=g, device="cuda") * 0.5).bfloat16()
    q = (torch.randn(len(lens), hq, d, generator=g, device="cuda") * 0.5).bfloat16()
    cos, sin = ao.rope_tables(pt.shape[1] * 64, d, 500000.0)
    return pt, q, k, v, torch.tensor(lens, dtype=torch.int32, device="cuda"), \
        torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _close(a, b):
    err = (a.float() - b.float()).abs()
    return err.max().item() <= HALF_MAX and err.mean().item() <= HALF_MEAN


@pytest.mark.parametrize("split", [0, 3])
def test_noalloc_decode_matches_the_allocating_entry(cuda, split):
    lens = [3000, 700, 64, 1500, 9000]
    pt, q, k, v, lens_t, cos, sin = _case(lens, 64, 8, 128, seed=11)
    call = ba.DecodeCall(pt, q, k, v, lens_t, cos, sin, split_blocks=split)
    assert call.plan["max_splits"] > 1          # the scratch is really used
    want = call.launch().clone()
    lib = _native.lib()
    for _ in range(2):                          # two calls in a row share the array
        out = torch.full_like(want, float("nan"))
        args = ba._decode_args(*call._keep[:8], call._keep[8], call._keep[9], False, None,
                               split, "auto", out, None, None)
        _native.check(lib.ouro_paged_decode_noalloc(ctypes.byref(args), _stream()),
                      "noalloc decode")
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        assert _close(out, want)


def test_noalloc_refuses_an_explicit_split_that_does_not_fit(cuda):
    lens = [600] * 256                          # 256 x 64 heads x 10 chunks of partials
    pt, q, k, v, lens_t, cos, sin = _case(lens, 64, 8, 128, seed=5)
    call = ba.DecodeCall(pt, q, k, v, lens_t, cos, sin, split_blocks=1)
    args = ba._decode_args(*call._keep[:8], call._keep[8], call._keep[9], False, None, 1,
                           "auto", torch.empty_like(q), None, None)
    rc = _native.lib().ouro_paged_decode_noalloc(ctypes.byref(args), _stream())
    assert rc == _native.OURO_EINVAL
    assert "static scratch" in _native.last_error()
    # with split_blocks = 0 it picks larger chunks that fit, and matches
    want = ba.DecodeCall(pt, q, k, v, lens_t, cos, sin).launch().clone()
    out = torch.empty_like(want)
    args = ba._decode_args(*call._keep[:8], call._keep[8], call._keep[9], False, None, 0,
                           "auto", out, None, None)
    _native.check(_native.lib().ouro_paged_decode_noalloc(ctypes.byref(args), _stream()),
                  "noalloc decode")
    torch.cuda.synchronize()
    assert _close(out, want)


def test_noalloc_replans_when_the_default_plan_does_not_fit(cuda):
    """256 sequences of 94 blocks on the split-K kernel: its default plan's partials
    (about 51 MB) exceed the 32 MiB array, so the entry point re-plans with fewer,
    larger chunks; the rows still match the allocating entry point."""
    lens = [6000] * 256
    pt, q, k, v, lens_t, cos, sin = _case(lens, 64, 8, 128, seed=6)
    call = ba.DecodeCall(pt, q, k, v, lens_t, cos, sin, total_blocks=256 * 94,
                         max_seq_blocks=94, kernel="tc")
    assert call.plan["workspace_bytes"] > 32 << 20   # the default plan does not fit
    want = call.launch().clone()
    for _ in range(2):
        out = torch.full_like(want, float("nan"))
        args = ba._decode_args(*call._keep[:8], call._keep[8], call._keep[9], False, None, 0,
                               "tc", out, None, None, 256 * 94, 94)
        _native.check(_native.lib().ouro_paged_decode_noalloc(ctypes.byref(args), _stream()),
                      "noalloc decode")
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        assert _close(out, want)
