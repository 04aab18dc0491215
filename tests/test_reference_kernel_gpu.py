"""This repository's block_attention against the reference's own Triton kernel, on the GPU.

The reference's Triton kernel (reference src/kernels/block_attention.py:188-342,
launched by its wrapper at :368-527) runs here from the unmodified install in
baseline/_ref (loaded by tests/reference_kernel.py). Both implementations get
identical inputs; every valid row (position < seq_len) of every sequence and
head is compared, within max-abs 2e-2 and mean-abs 2e-3 (the fp16/bf16
tolerance; the reference's fp32 tl.dot runs as TF32, so its fp32 results are
held to the same bound). Cases: the reference's own GPU-test shape with and
without bias + block mask (fp32, fp16), the CPU-runnable decode batch (4
sequences, lens {64, 130, 200, 511}, H 8, D 64, fp32) and a slice of the fp16
MHA shape (H 32, D 128) with a Table-1 token scope passed as a -inf bias.
"""

import numpy as np
import pytest
import torch

import cases
import reference_kernel
from src.block_table import BlockTable
from src.kernels import block_attention as ba
from src.scoping_mask import scope_bias

pytestmark = pytest.mark.gpu
MAX_ABS, MEAN_ABS = 2e-2, 2e-3


@pytest.fixture(scope="module")
def ref():
    return reference_kernel.load()


def _run_both(ref, c, **kw):
    pt = torch.tensor(c["rows"], dtype=torch.int32).cuda()
    args = (pt, c["q_cache"].cuda(), c["k_cache"].cuda(), c["v_cache"].cuda(),
            torch.tensor(c["lens"], dtype=torch.int32).cuda(), c["cos"].cuda(), c["sin"].cuda())
    want = ref.block_attention(*args, **kw)
    got = ba.block_attention(*args, **kw)
    torch.cuda.synchronize()
    assert got.shape == want.shape and got.dtype == want.dtype
    errs = []
    for s, n in enumerate(c["lens"]):
        e = (got[s, :, :n].float() - want[s, :, :n].float()).abs()
        errs.append(e.reshape(-1))
    e = torch.cat(errs)
    assert torch.isfinite(want[:, :, :max(c["lens"])].float()).all()
    return float(e.max()), float(e.mean())


@pytest.mark.parametrize("name", ["bm", "plain", "f16"])
def test_matches_reference_triton_on_its_own_test_shape(cuda, ref, name):
    seed = {"bm": 1234, "plain": 77, "f16": 5}[name]
    dt = torch.float16 if name == "f16" else torch.float32
    c = cases.small_full_case(torch, BlockTable, seed, dtype=dt)
    kw = {}
    if name == "bm":
        gen = torch.Generator().manual_seed(seed + 1)
        bias = torch.randn(1, 2, max(c["lens"]), max(c["lens"]), generator=gen) * 0.25
        scope = torch.randint(0, 2, (2, 3, 3), generator=gen) | torch.eye(3, dtype=torch.int64)
        kw = dict(bias=bias.cuda(), mask=scope.to(torch.int8).cuda())
    mx, mean = _run_both(ref, c, **kw)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


def test_matches_reference_triton_on_the_cpu_decode_batch(cuda, ref):
    c = cases.config1_case(torch, BlockTable)
    mx, mean = _run_both(ref, c)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


def test_matches_reference_triton_with_a_token_scope_bias(cuda, ref):
    lens = [700, 1100]
    bt, heads, rows = cases.scattered_chains(BlockTable, 64, lens, 21)
    q, k, v = cases.paged_caches(torch, 21, 64, 32, 128, 0.5, torch.float16)
    cos, sin = cases.rope_tables_torch(torch, len(rows[0]) * 64, 128, 10000.0)
    T = max(lens)
    bias = torch.zeros(len(lens), 1, T, T)
    for s, n in enumerate(lens):
        spans = cases.segment_spans(n, 100 + s)
        bias[s, 0, :n, :n] = torch.from_numpy(scope_bias(spans))
    c = dict(lens=lens, rows=rows, q_cache=q, k_cache=k, v_cache=v, cos=cos, sin=sin)
    mx, mean = _run_both(ref, c, bias=bias.cuda())
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("with_mask", [False, True])
def test_matches_reference_triton_on_the_tensor_core_path(cuda, ref, dtype, with_mask):
    """Head_dim 128, no bias: this repository's call runs on the tcgen05 kernel."""
    lens = [700, 1100, 64, 257]
    bt, heads, rows = cases.scattered_chains(BlockTable, 64, lens, 5)
    q, k, v = cases.paged_caches(torch, 5, 64, 8, 128, 0.5, dtype)
    cos, sin = cases.rope_tables_torch(torch, len(rows[0]) * 64, 128, 10000.0)
    c = dict(lens=lens, rows=rows, q_cache=q, k_cache=k, v_cache=v, cos=cos, sin=sin)
    kw = {}
    if with_mask:
        qb = -(-max(lens) // 64)
        m = (torch.rand(len(lens), qb, qb, generator=torch.Generator().manual_seed(2)) < 0.6)
        kw = dict(mask=(m.to(torch.int8) | torch.eye(qb, dtype=torch.int8)).cuda())
    mx, mean = _run_both(ref, c, **kw)
    assert mx <= MAX_ABS and mean <= MEAN_ABS, (mx, mean)
