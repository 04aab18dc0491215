"""Serving layer: the reference's Supervisor/Worker contract and the sharded data plane.

Control-plane behaviours re-asserted from the reference (src/serving.py:1-58,
its tests/test_serving.py and scripts/demo_serving.py invariants): stateless
workers, crash -> chain freed first -> safe queue, FIFO drain on fresh
chains, zero block leak, [EXPAND] bookkeeping. Data-plane bookkeeping (pools,
LPT placement, chain growth, page-table slices) runs on CPU tensors here;
the GPU decode through the Supervisor is in test_serving_gpu.py.
"""

import pytest
import torch

from src.block_table import BLOCK_SIZE, BlockTable
from src.serving import (SAFE_QUEUE_PREFIX, KVPool, Supervisor, Worker, WorkerCrash,
                         lpt_placement, pool_blocks_for)


def test_worker_is_a_pure_transform():
    w = Worker("w1")
    w.start()
    before = dict(vars(w))
    assert w.process("abc") == "ok:cba" == w.process("abc")
    assert vars(w) == before
    w.kill()
    with pytest.raises(WorkerCrash):
        w.process("x")


def test_fail_next_is_one_shot():
    w = Worker("w", fail_next=True)
    w.start()
    with pytest.raises(WorkerCrash):
        w.process("boom")
    assert w.alive is False


def test_supervisor_owns_table_and_workers_hold_nothing():
    sup = Supervisor()
    sup.add_worker("w1")
    assert isinstance(sup.block_table, BlockTable) and sup.kv_cache == {}
    assert not hasattr(sup.workers["w1"], "block_table")
    assert sup.table_op(lambda bt: bt) is sup.block_table
    with pytest.raises(RuntimeError, match="already exists"):
        sup.add_worker("w1")


def test_submit_allocates_by_utf8_bytes_and_records_ownership():
    sup = Supervisor(max_blocks=32)
    sup.add_worker("w")
    free0 = sup.block_table.num_free
    assert sup.submit("hello") == "ok:olleh"
    assert sup.last_request_id == 1 and sup.block_table.num_free == free0 - 1
    big = "é" * 40                        # 80 UTF-8 bytes -> 2 blocks
    sup.submit(big)
    assert sup.block_table.chain_len(sup.kv_cache[2]) == 2
    assert sup.chain_capacity[2] == 2 * BLOCK_SIZE


def test_crash_frees_chain_then_queues_and_drain_reserves_fresh():
    sup = Supervisor(max_blocks=16)
    sup.add_worker("w0", fail_next=True)
    free0 = sup.block_table.num_free
    res = sup.submit("payload-" * 20)
    assert res == SAFE_QUEUE_PREFIX + "payload-" * 20
    assert sup.block_table.num_free == free0          # zero leak
    assert sup.kv_cache == {} and sup.safe_queue == ["payload-" * 20]
    with pytest.raises(RuntimeError, match="no alive worker"):
        sup.submit("x")
    assert sup.drain_safe_queue() == [SAFE_QUEUE_PREFIX + "payload-" * 20]   # still queued
    assert sup.health_pass() == ["w0"]
    sup.restart("w0")
    out = sup.drain_safe_queue()
    assert out == ["ok:" + ("payload-" * 20)[::-1]] and sup.safe_queue == []
    assert sup.last_request_id == 2                    # ids never reused


def test_expand_and_release():
    sup = Supervisor(max_blocks=16)
    sup.add_worker("w")
    sup.submit("abc")
    tail = sup.expand_request(1, extra_bytes=200)    # ceil(200/64) = 4 blocks
    assert sup.block_table.chain_len(sup.kv_cache[1]) == 5
    assert sup.block_table.chain_tail(sup.kv_cache[1]) == tail
    assert sup.chain_capacity[1] == 5 * 64
    for bad in (0, -3, True, 1.5):
        with pytest.raises(RuntimeError):
            sup.expand_request(1, bad)
    free = sup.block_table.num_free
    sup.release(1)
    assert sup.block_table.num_free == free + 5
    with pytest.raises(RuntimeError, match="already-released"):
        sup.release(1)


def test_lpt_placement_balances_tokens():
    lens = [9000, 30000, 12000, 31000, 8200, 20000, 17000, 25000]
    loads = [0, 0, 0, 0]
    where = lpt_placement(lens, loads)
    assert sum(loads) == sum(lens)
    assert max(loads) - min(loads) <= max(lens)
    # the longest sequence lands on pool 0 (empty, lowest index)
    assert where[lens.index(31000)] == 0


def _cpu_pools(n, blocks=64):
    return [KVPool(device=torch.device("cpu"), num_blocks=blocks, kv_heads=2, head_dim=16,
                   dtype=torch.float32, max_positions=blocks * 64) for _ in range(n)]


def test_admit_reserve_shard_finish_bookkeeping():
    sup = Supervisor(pools=_cpu_pools(2))
    rids = sup.admit_many([500, 130, 1000, 64])
    assert len({sup.seqs[r].pool for r in rids}) == 2
    for r, n in zip(rids, [500, 130, 1000, 64]):
        sup.reserve(r, n)
        sup.seqs[r].length = n
    shards = sup.shard(rids)
    for p, (rs, pt, lens) in shards.items():
        table = sup.pools[p].table
        for row, r, ln in zip(pt, rs, lens):
            chain = list(table.walk(sup.seqs[r].head))
            assert row[:len(chain)].tolist() == chain and ln == sup.seqs[r].length
            assert len(chain) * 64 >= ln
    sup.reserve(rids[1], 200)                     # grows 3 -> 6 blocks at the tail
    st = sup.seqs[rids[1]]
    assert sup.pools[st.pool].table.chain_len(st.head) == -(-(130 + 200) // 64)
    free = [p.table.num_free for p in sup.pools]
    for r in rids:
        sup.finish(r)
    assert [p.table.num_free for p in sup.pools] == [64, 64] and sum(free) < 128


def test_decode_tables_kept_between_calls_and_refreshed_by_row():
    """decode_step's per-pool page tables: exported once, then only the rows whose chain
    grew are rewritten; a chain longer than the kept width (steps of 32 blocks) brings a
    full export; a finished sequence drops the kept tables."""
    sup = Supervisor(pools=_cpu_pools(1, blocks=256))
    rids = sup.admit_many([100, 64, 1900])
    for r, n in zip(rids, [100, 64, 1900]):
        sup.seqs[r].length = n

    def rows_ok(pt):
        table = sup.pools[0].table
        for row, r in zip(pt, rids):
            chain = list(table.walk(sup.seqs[r].head))
            assert row[:len(chain)].tolist() == chain
            assert (row[len(chain):] == -1).all()

    pt, widest = sup._device_table(0, rids)
    assert tuple(pt.shape) == (3, 32) and widest == 30
    rows_ok(pt)
    sup.reserve(rids[1], 10)                      # 64 -> 74 tokens: one more block
    pt2, _ = sup._device_table(0, rids)
    assert pt2.data_ptr() == pt.data_ptr()        # same kept table, one row rewritten
    rows_ok(pt2)
    sup.reserve(rids[2], 200)                     # 1900 -> 2100 tokens: 33 blocks > 32
    pt3, widest = sup._device_table(0, rids)
    assert tuple(pt3.shape) == (3, 64) and widest == 33
    rows_ok(pt3)
    sup.finish(rids[0])
    assert sup._tables == {}


def test_admission_refuses_when_no_pool_has_room():
    sup = Supervisor(pools=_cpu_pools(2, blocks=4))
    sup.admit(4 * 64)
    sup.admit(4 * 64)
    with pytest.raises(RuntimeError, match="insufficient free blocks"):
        sup.admit(64)


def test_pool_sizing():
    assert pool_blocks_for([64, 65], headroom=0.0) == 4
