"""Continuous-batching scheduler of the serving trace, on the CPU.

The engine runs against a stand-in backend that records every prefill and
decode call and checks what the GPU backend relies on: page-table rows cover
the positions written, chunks stay within their budgets, decode positions
advance one token at a time. The native allocator is the real one.
"""

import math
import random

import numpy as np
import pytest

from src.block_table import BLOCK_SIZE, BlockTable, PAD_ID
from src.engine import Engine, Request, make_trace, random_segments, shard_requests
from src.scoping_mask import GLOBAL, LOCAL, token_scope


class RecordingBackend:
    def __init__(self, table, engine=None):
        self.table = table
        self.engine = engine
        self.admitted, self.released = [], []
        self.pos = {}            # rid -> next position expected
        self.prefill_calls = self.decode_calls = 0

    def admit(self, r, blocks):
        assert blocks == list(self.table.walk(r.head)) and len(blocks) == r.blocks
        self.admitted.append(r.rid)
        self.pos[r.rid] = 0

    def release(self, r):
        self.released.append(r.rid)

    def _rows_cover(self, reqs, pt, ends):
        for i, (r, e) in enumerate(zip(reqs, ends)):
            row = [b for b in pt[i] if b != PAD_ID]
            assert row == list(self.table.walk(r.head))
            assert len(row) * BLOCK_SIZE >= e, (r.rid, len(row), e)

    def prefill(self, reqs, starts, counts):
        self.prefill_calls += 1
        self._rows_cover(reqs, self.engine.page_table(reqs), starts + counts)
        for r, s, c in zip(reqs, starts, counts):
            assert s == self.pos[r.rid] and 0 < c
            self.pos[r.rid] = s + c
        return [(r.rid * 31 + int(s)) % 97 for r, s in zip(reqs, starts)]

    def decode(self, reqs, pos):
        self.decode_calls += 1
        self._rows_cover(reqs, self.engine.page_table(reqs), pos + 1)
        for r, p in zip(reqs, pos):
            assert p == self.pos[r.rid] == r.prompt_len + r.generated - 1
            assert p < r.total
            self.pos[r.rid] = p + 1
        return [(r.rid + int(p)) % 97 for r, p in zip(reqs, pos)]


class FakeClock:
    def __init__(self, dt):
        self.t, self.dt = 0.0, dt

    def __call__(self):
        self.t += self.dt
        return self.t

    def sleep(self, s):
        self.t += s


def test_trace_shape():
    tr = make_trace(4000, rate=64.0, median=2048, sigma=1.0, lo=128, hi=16384, max_new=256, seed=1)
    lens = np.array([r.prompt_len for r in tr])
    assert lens.min() >= 128 and lens.max() <= 16384
    assert 1800 < np.median(lens) < 2300
    gaps = np.diff([0.0] + [r.arrival for r in tr])
    assert abs(gaps.mean() - 1 / 64.0) < 0.002
    r = tr[0]
    tags, start, end = token_scope(r.spans)
    assert len(tags) == r.prompt_len + 256 and tags[0] == 1


def test_random_segments_partition():
    rng = random.Random(3)
    for total in (1, 31, 32, 513, 5000):
        sp = random_segments(rng, total)
        assert sp[0][0] == 0 and sp[-1][1] == total and sp[0][2] == GLOBAL
        assert all(a[1] == b[0] for a, b in zip(sp, sp[1:]))
        assert all(e - s <= 512 for s, e, _ in sp)
        assert {sc for _, _, sc in sp} <= {GLOBAL, LOCAL}


@pytest.mark.parametrize("pool_blocks,chunk,budget", [(4000, 256, 1024), (60, 128, 300)])
def test_engine_serves_every_request_and_frees_every_block(pool_blocks, chunk, budget):
    tr = make_trace(40, rate=200.0, median=300, sigma=0.8, lo=16, hi=1500, max_new=7, seed=5)
    tr[3].max_new = 1                      # a request that finishes at its prefill
    table = BlockTable(pool_blocks)
    be = RecordingBackend(table)
    eng = Engine(table, be, chunk=chunk, prefill_tokens=budget, slots=64)
    be.engine = eng
    clock = FakeClock(0.002)
    st = eng.run(tr, clock=clock, sleep=clock.sleep)
    assert st["requests"] == 40 and st["generated_tokens"] == sum(r.max_new for r in tr)
    assert table.num_free == pool_blocks and eng.idle
    assert sorted(be.released) == sorted(be.admitted) == list(range(40))
    assert be.admitted == sorted(be.admitted, key=lambda i: (tr[i].arrival, i))  # arrival order
    for r in tr:
        assert r.admit_time >= r.arrival and r.finish_time >= r.first_token_time >= r.admit_time
        assert be.pos[r.rid] == r.prompt_len + r.max_new - 1
    assert st["peak_blocks"] <= pool_blocks


def test_engine_timer_gives_token_times_of_the_producing_steps():
    """With a timer (no per-step sync) first-token and finish times are the marks of the
    steps that produced those tokens, read after the run."""
    tr = make_trace(12, rate=500.0, median=200, sigma=0.5, lo=16, hi=800, max_new=5, seed=9)
    table = BlockTable(400)
    be = RecordingBackend(table)
    eng = Engine(table, be, chunk=128, prefill_tokens=256, slots=32)
    be.engine = eng

    class StepTimer:                      # mark i resolves to 10 + i seconds
        def __init__(self):
            self.marks, self.synced = 0, False

        def start(self):
            self.marks = 0

        def mark(self):
            self.marks += 1
            return self.marks - 1

        def sync(self):
            self.synced = True

        def seconds(self, m):
            return 10.0 + m

    timer = StepTimer()
    clock = FakeClock(0.001)
    st = eng.run(tr, clock=clock, sleep=clock.sleep, timer=timer)
    assert timer.synced and timer.marks == eng.steps == st["steps"]
    for r in tr:
        assert r.first_token_time == 10.0 + r.first_token_step
        assert r.finish_time == 10.0 + r.finish_step
        # prefill completes at one step; the remaining max_new - 1 tokens take one step each
        assert r.finish_step - r.first_token_step >= r.max_new - 1


def test_engine_prefill_respects_chunk_and_budget():
    tr = [Request(i, 0.0, L, 3, random_segments(random.Random(i), L + 3))
          for i, L in enumerate([1000, 70, 2500, 5])]
    table = BlockTable(500)
    seen = []

    class B(RecordingBackend):
        def prefill(self, reqs, starts, counts):
            seen.append(list(counts))
            return super().prefill(reqs, starts, counts)

    be = B(table)
    eng = Engine(table, be, chunk=512, prefill_tokens=900)
    be.engine = eng
    clock = FakeClock(0.001)
    eng.run(tr, clock=clock, sleep=clock.sleep)
    assert all(max(c) <= 512 and sum(c) <= 900 for c in seen)
    assert sum(map(sum, seen)) == 1000 + 70 + 2500 + 5


def test_admission_waits_for_free_blocks():
    big = Request(0, 0.0, 60 * 64, 4, random_segments(random.Random(0), 60 * 64 + 4))
    small = Request(1, 0.0, 64, 4, random_segments(random.Random(1), 68))
    table = BlockTable(62)                 # room for big (61 blocks) but not both at once
    be = RecordingBackend(table)
    eng = Engine(table, be, chunk=4096, prefill_tokens=8192)
    be.engine = eng
    eng.submit([big, small])
    eng.step(0.0)
    assert [r.rid for r in eng.running] == [0] and len(eng.waiting) == 1
    clock = FakeClock(0.001)
    eng.run([], clock=clock, sleep=clock.sleep)
    assert small.admit_time >= big.finish_time and table.num_free == 62


def test_shard_requests_lpt():
    tr = make_trace(100, rate=64.0, median=2048, sigma=1.0, lo=128, hi=16384, max_new=256, seed=2)
    shards = shard_requests(tr, 8)
    assert sorted(r.rid for s in shards for r in s) == list(range(100))
    loads = [sum(r.total for r in s) for s in shards]
    assert max(loads) - min(loads) <= max(r.total for r in tr)
    for s in shards:
        assert [r.arrival for r in s] == sorted(r.arrival for r in s)
