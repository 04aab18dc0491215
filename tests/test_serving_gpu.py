"""Serving data plane on the GPU: pools, K/V append, sharded decode, worker crash.

Two pools (on the same GPU here; one per GPU in deployment) own the caches;
sequences are admitted with LPT placement, their prompt K/V written through
the append kernel, then one decode step runs shard by shard through stateless
workers and is checked against the oracle over the same cache contents.
"""

import numpy as np
import pytest
import torch

from oracle import attention_oracle as ao
from src.serving import KVPool, Supervisor

pytestmark = pytest.mark.gpu


def _pools(n, blocks=96, hkv=2, d=128, dtype=torch.bfloat16):
    return [KVPool(device=torch.device("cuda", 0), num_blocks=blocks, kv_heads=hkv, head_dim=d,
                   dtype=dtype, max_positions=blocks * 64, rope_base=500000.0)
            for _ in range(n)]


def _oracle_rows(sup, rids, q):
    outs = []
    for i, r in enumerate(rids):
        st = sup.seqs[r]
        pool = sup.pools[st.pool]
        row = np.asarray([pool.table.page_table_row(st.head)], np.int32)
        k = pool.k_cache.float().cpu().numpy()
        v = pool.v_cache.float().cpu().numpy()
        o = ao.decode_attention(row, q[i:i + 1].float().cpu().numpy(), k, v, [st.length],
                                pool.cos.cpu().numpy(), pool.sin.cpu().numpy())
        outs.append(o[0])
    return np.stack(outs)


def test_append_then_sharded_decode_matches_oracle(cuda):
    sup = Supervisor(pools=_pools(2))
    lens = [700, 64, 1300, 250, 999]
    rids = sup.admit_many(lens)
    assert {sup.seqs[r].pool for r in rids} == {0, 1}
    g = torch.Generator(device="cuda").manual_seed(0)
    L = max(lens)
    k_new = (torch.randn(len(lens), 2, L, 128, generator=g, device="cuda") * 0.5).bfloat16()
    v_new = (torch.randn(len(lens), 2, L, 128, generator=g, device="cuda") * 0.5).bfloat16()
    sup.append_kv(rids, k_new, v_new, counts=lens)
    assert [sup.seqs[r].length for r in rids] == lens
    # the decoded token's own K/V goes in first, then the step attends over it
    k1 = (torch.randn(len(lens), 2, 1, 128, generator=g, device="cuda") * 0.5).bfloat16()
    v1 = (torch.randn(len(lens), 2, 1, 128, generator=g, device="cuda") * 0.5).bfloat16()
    sup.append_kv(rids, k1, v1)
    q = (torch.randn(len(lens), 16, 128, generator=g, device="cuda") * 0.5).bfloat16()
    out = sup.decode_step(rids, q)
    want = _oracle_rows(sup, rids, q)
    err = np.abs(out.float().cpu().numpy() - want)
    assert err.max() < 2e-2 and err.mean() < 2e-3, (err.max(), err.mean())
    # appended tokens landed where the page table says (spot-check one token)
    st = sup.seqs[rids[2]]
    pool = sup.pools[st.pool]
    row = pool.table.page_table_row(st.head)
    tok = 1299
    assert torch.equal(pool.k_cache[row[tok // 64], :, tok % 64], k_new[2, :, tok])


def test_crashed_worker_is_replaced_and_the_step_completes(cuda):
    sup = Supervisor(pools=_pools(1))
    rids = sup.admit_many([300, 500])
    g = torch.Generator(device="cuda").manual_seed(1)
    kv = (torch.randn(2, 2, 500, 128, generator=g, device="cuda") * 0.5).bfloat16()
    sup.append_kv(rids, kv, kv.flip(2), counts=[300, 500])
    q = (torch.randn(2, 16, 128, generator=g, device="cuda") * 0.5).bfloat16()
    ref = sup.decode_step(rids, q).clone()
    w = sup._gpu_worker(0)
    w._fail_next = True                      # the next call dies mid-request
    out = sup.decode_step(rids, q)
    assert torch.equal(out, ref)             # pools untouched, shard re-dispatched
    assert sup._gpu_workers[0] is not w      # a fresh worker took over


def test_finish_returns_every_block(cuda):
    sup = Supervisor(pools=_pools(2, blocks=40))
    rids = sup.admit_many([640, 64, 1000])
    for r in rids:
        sup.reserve(r, 64)
    for r in rids:
        sup.finish(r)
    assert [p.table.num_free for p in sup.pools] == [40, 40]


def test_decode_loop_across_block_boundaries_matches_oracle(cuda):
    """decode_step keeps each pool's page table on the device between calls and refreshes
    only the rows whose chain grew (and the whole table when the longest chain outgrows
    the kept width, 32 blocks): a few decode steps whose appended tokens cross block
    boundaries, each checked against the oracle."""
    sup = Supervisor(pools=_pools(2, blocks=160))
    lens = [63, 127, 2045, 64, 300]
    rids = sup.admit_many(lens)
    g = torch.Generator(device="cuda").manual_seed(7)
    L = max(lens)
    k_new = (torch.randn(len(lens), 2, L, 128, generator=g, device="cuda") * 0.5).bfloat16()
    v_new = (torch.randn(len(lens), 2, L, 128, generator=g, device="cuda") * 0.5).bfloat16()
    sup.append_kv(rids, k_new, v_new, counts=lens)
    for step in range(4):
        n_new = 1 if step < 3 else 5     # the last step takes the 2045-token chain past 32 blocks
        k1 = (torch.randn(len(lens), 2, n_new, 128, generator=g, device="cuda") * 0.5).bfloat16()
        v1 = (torch.randn(len(lens), 2, n_new, 128, generator=g, device="cuda") * 0.5).bfloat16()
        sup.append_kv(rids, k1, v1)
        q = (torch.randn(len(lens), 16, 128, generator=g, device="cuda") * 0.5).bfloat16()
        out = sup.decode_step(rids, q)
        want = _oracle_rows(sup, rids, q)
        err = np.abs(out.float().cpu().numpy() - want)
        assert err.max() < 2e-2 and err.mean() < 2e-3, (step, err.max(), err.mean())
    assert sup.seqs[rids[2]].length == 2045 + 3 + 5 and sup.seqs[rids[2]].blocks == 33
    assert sup.seqs[rids[0]].blocks == 2 and sup.seqs[rids[3]].blocks == 2
