"""Serving engine on one GPU: continuous batching with the real kernels.

A small trace runs step by step through the stand-in model on the tensor-core
prefill and decode kernels. After prefill and decode steps the attention
output of the whole batch (token scope, positions and page tables as the
engine built them) is checked against the oracle on the cache as it stands
(max-abs 2e-2, mean-abs 2e-3, bf16); at the end every request has its output
tokens and every block is back in the pool.
"""

import numpy as np
import pytest
import torch

from oracle import attention_oracle as ao
from src.engine import Engine, StandInBackend, make_trace
from src.serving import KVPool

pytestmark = pytest.mark.gpu


def test_engine_trace_matches_oracle_and_frees_pool(cuda):
    tr = make_trace(24, rate=400.0, median=300, sigma=0.9, lo=16, hi=1200, max_new=6, seed=11)
    pool = KVPool(device=torch.device("cuda", 0), num_blocks=160, kv_heads=8, head_dim=128,
                  dtype=torch.bfloat16, max_positions=2048, rope_base=500000.0)
    be = StandInBackend(pool, 32, max_total=2048, slots=64, seed=1)
    eng = Engine(pool.table, be, chunk=256, prefill_tokens=1024, slots=64)
    eng.submit(tr)
    checked, checked_prefill, now = 0, 0, 0.0
    be.last_prefill = None
    cos, sin = pool.cos.cpu().numpy(), pool.sin.cpu().numpy()
    while not eng.idle:
        steps = eng.steps
        be.last_decode = None
        eng.step(now)
        if be.last_prefill is not None and checked_prefill < 2:
            pt, q, st, lens, scope, out = be.last_prefill
            torch.cuda.synchronize()
            want = ao.prefill_attention(pt.cpu().numpy(), q.float().cpu().numpy(),
                                        pool.k_cache.float().cpu().numpy(),
                                        pool.v_cache.float().cpu().numpy(), st.cpu().numpy(),
                                        lens.cpu().numpy(), cos, sin, causal=True,
                                        scope_tags=scope[0].cpu().numpy(),
                                        scope_lo=scope[1].cpu().numpy(),
                                        scope_hi=scope[2].cpu().numpy())
            got = out.float().cpu().numpy()
            for i, n in enumerate((lens - st).tolist()):
                err = np.abs(got[i, :, :n] - want[i, :, :n])
                assert err.max() <= 2e-2 and err.mean() <= 2e-3, ("prefill", err.max(), err.mean())
            checked_prefill += 1
            be.last_prefill = None
        now += 0.003
        if be.last_decode is not None and checked < 4 and eng.steps > steps:
            pt, q, lens, tags, span, out = be.last_decode
            torch.cuda.synchronize()
            want = ao.decode_attention(pt.cpu().numpy(), q.float().cpu().numpy(),
                                       pool.k_cache.float().cpu().numpy(),
                                       pool.v_cache.float().cpu().numpy(),
                                       lens.cpu().numpy(), cos, sin,
                                       scope_tags=tags.cpu().numpy(),
                                       scope_span=span.cpu().numpy())
            err = np.abs(out.float().cpu().numpy() - want)
            assert err.max() <= 2e-2 and err.mean() <= 2e-3, (err.max(), err.mean())
            checked += 1
        assert eng.steps < 10000
    assert checked >= 3 and checked_prefill == 2
    assert len(eng.finished) == 24 and all(r.generated == r.max_new for r in eng.finished)
    assert pool.table.num_free == 160
    assert be.kv_bytes > 0 and be.attn_ms() > 0
