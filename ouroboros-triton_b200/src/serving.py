"""Supervisor-Worker serving layer.

Two layers in one module:

1. The reference's control-plane contract, kept call-for-call
   (src/serving.py:65-329): ``Supervisor`` owns THE block table and the KV
   bookkeeping (``kv_cache``: request id -> chain head, ``chain_capacity``),
   ``Worker`` is stateless (``process`` mutates nothing), a ``WorkerCrash``
   frees the request's chain before the request goes to the Phase-1 safe
   queue, ``drain_safe_queue`` replays FIFO on fresh chains.

2. The GPU data plane the reference does not have: the Supervisor also owns
   one :class:`KVPool` per GPU (paged K/V caches plus that GPU's native block
   allocator) and shards whole sequences across them by token count
   (longest-processing-time placement). A decode step hands each pool's
   (query shard, page-table slice, lengths) to a stateless :class:`Worker`
   bound to that GPU; the outputs come back to the Supervisor's device
   (peer copies in one process; NCCL gather across processes, see
   :mod:`src.dist`). Workers never hold a pool, a table or a cache.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Callable

from .block_table import BLOCK_SIZE, BlockTable

#: Prefix marking a request degraded to the Phase-1 Safe Queue by submit().
SAFE_QUEUE_PREFIX = "safe-queued:"


class WorkerCrash(RuntimeError):
    """A worker died mid-request (stands in for a kernel crash taking the worker down)."""


class Worker:
    """Stateless, restartable executor (reference src/serving.py:72-117).

    ``process`` is a pure transform of the request string; ``decode`` runs one
    paged-decode shard on the worker's GPU from arguments alone. Neither writes
    any attribute: a restart is "drop the object, build a new one".
    """

    def __init__(self, worker_id, fail_next: bool = False, device=None):
        self.worker_id = worker_id
        self.alive = False
        self._fail_next = bool(fail_next)
        self.device = device

    def start(self) -> None:
        self.alive = True

    def kill(self) -> None:
        self.alive = False

    def _check_alive(self) -> None:
        if not self.alive:
            raise WorkerCrash(f"worker {self.worker_id!r} is dead (segfaulted)")
        if self._fail_next:
            self._fail_next = False  # one-shot
            self.kill()
            raise WorkerCrash(f"worker {self.worker_id!r} simulated segfault (fail_next)")

    def process(self, request: str) -> str:
        """Deterministic stand-in for one inference step: ``"ok:" + reversed request``."""
        self._check_alive()
        return f"ok:{request[::-1]}"

    def decode(self, k_cache, v_cache, cos, sin, q, page_table, seq_lens, **kw):
        """One decode shard on this worker's GPU; every input is an argument."""
        self._check_alive()
        from .kernels.block_attention import block_attention_decode

        return block_attention_decode(page_table, q, k_cache, v_cache, seq_lens, cos, sin,
                                      validate=False, **kw)


@dataclass
class KVPool:
    """Supervisor-owned KV storage on one GPU: paged caches + its allocator."""

    device: object
    num_blocks: int
    kv_heads: int
    head_dim: int
    dtype: object
    max_positions: int
    rope_base: float = 10000.0
    table: BlockTable = field(init=False)
    k_cache: object = field(init=False)
    v_cache: object = field(init=False)
    cos: object = field(init=False)
    sin: object = field(init=False)

    def __post_init__(self):
        import torch

        self.table = BlockTable(self.num_blocks)
        shape = (self.num_blocks, self.kv_heads, BLOCK_SIZE, self.head_dim)
        self.k_cache = torch.zeros(shape, dtype=self.dtype, device=self.device)
        self.v_cache = torch.zeros(shape, dtype=self.dtype, device=self.device)
        half = self.head_dim // 2
        inv = 1.0 / (float(self.rope_base) ** (torch.arange(half, dtype=torch.float64) * 2.0
                                                / self.head_dim))
        ang = torch.arange(self.max_positions, dtype=torch.float64)[:, None] * inv[None, :]
        self.cos = torch.cos(ang).float().to(self.device)
        self.sin = torch.sin(ang).float().to(self.device)


@dataclass
class SeqState:
    pool: int
    head: int
    length: int  # tokens whose K/V are in the cache
    blocks: int = 0  # the chain's length in blocks


def lpt_placement(lengths, loads) -> list[int]:
    """Longest-processing-time placement of sequences onto pools.

    Sequences are taken longest first and each goes to the pool with the
    least token load so far (lowest index on ties). Returns the pool index
    per sequence, in the input order; ``loads`` is updated in place.
    """
    order = sorted(range(len(lengths)), key=lambda i: (-lengths[i], i))
    out = [0] * len(lengths)
    for i in order:
        p = min(range(len(loads)), key=lambda j: (loads[j], j))
        out[i] = p
        loads[p] += lengths[i]
    return out


class Supervisor:
    """Owns the block tables, the KV pools and the request bookkeeping."""

    def __init__(self, max_blocks: int = 1024, pools: list[KVPool] | None = None,
                 device=None):
        self.block_table = BlockTable(max_blocks)
        self.kv_cache: dict = {}          # request_id -> chain head
        self.chain_capacity: dict = {}    # request_id -> capacity in tokens
        self.workers: dict = {}
        self.safe_queue: list[str] = []
        self._request_counter = 0
        # GPU data plane
        self.pools: list[KVPool] = list(pools or [])
        self.seqs: dict[int, SeqState] = {}
        self.device = device if device is not None else (
            self.pools[0].device if self.pools else None)
        self._gpu_workers: dict[int, Worker] = {}
        # decode_step's device page tables per (pool, rids): rows refreshed when a chain grows
        self._tables: dict = {}

    @property
    def last_request_id(self) -> int:
        return self._request_counter

    # -- chain lifecycle (reference src/serving.py:143-214) -----------------
    @staticmethod
    def _payload_blocks(request: str) -> int:
        """max(1, ceil(utf8_bytes / 64)) blocks for a request payload."""
        if not isinstance(request, str):
            raise RuntimeError(f"request must be str, got {type(request).__name__}")
        return max(1, -(-len(request.encode("utf-8")) // BLOCK_SIZE))

    def _free_chain(self, request_id) -> None:
        head = self.kv_cache.pop(request_id)
        self.chain_capacity.pop(request_id, None)
        self.block_table.free_chain(head)

    def expand_request(self, request_id, extra_bytes: int) -> int:
        """Grow a live chain by ceil(extra_bytes / 64) blocks; returns the new tail."""
        if request_id not in self.kv_cache:
            raise RuntimeError(f"unknown or already-released request id: {request_id!r}")
        if isinstance(extra_bytes, bool) or not isinstance(extra_bytes, int):
            raise RuntimeError(f"invalid extra_bytes: {extra_bytes!r}")
        if extra_bytes <= 0:
            raise RuntimeError(f"extra_bytes must be > 0, got {extra_bytes}")
        tail = self.block_table.chain_tail(self.kv_cache[request_id])
        for _ in range(-(-extra_bytes // BLOCK_SIZE)):
            tail = self.block_table.expand_chain(tail)
            self.chain_capacity[request_id] += BLOCK_SIZE
        return tail

    def release(self, request_id) -> None:
        if request_id not in self.kv_cache:
            raise RuntimeError(f"unknown or already-released request id: {request_id!r}")
        self._free_chain(request_id)

    # -- workforce (reference src/serving.py:218-243) ----------------------------
    def add_worker(self, worker_id, fail_next: bool = False) -> Worker:
        if worker_id in self.workers:
            raise RuntimeError(f"worker {worker_id!r} already exists")
        w = Worker(worker_id, fail_next=fail_next)
        w.start()
        self.workers[worker_id] = w
        return w

    def health_pass(self) -> list:
        return [wid for wid, w in self.workers.items() if not w.alive]

    def restart(self, worker_id) -> Worker:
        if worker_id not in self.workers:
            raise RuntimeError(f"unknown worker id: {worker_id!r}")
        fresh = Worker(worker_id, device=self.workers[worker_id].device)
        fresh.start()
        self.workers[worker_id] = fresh
        return fresh

    def table_op(self, fn: Callable[..., object], *args, **kwargs) -> object:
        """The only door from compute code into the Supervisor's table."""
        return fn(self.block_table, *args, **kwargs)

    # -- request routing (reference src/serving.py:257-329) ----------------------
    def submit(self, request: str, worker_id=None) -> str:
        if worker_id is not None:
            if worker_id not in self.workers:
                raise RuntimeError(f"unknown worker id: {worker_id!r}")
            candidates = [worker_id]
        else:
            candidates = list(self.workers)
        worker = next((self.workers[w] for w in candidates if self.workers[w].alive), None)
        if worker is None:
            raise RuntimeError("no alive worker available")
        self._request_counter += 1
        rid = self._request_counter
        head = self.block_table.allocate_chain(self._payload_blocks(request))
        self.kv_cache[rid] = head
        self.chain_capacity[rid] = self.block_table.chain_len(head) * BLOCK_SIZE
        try:
            return worker.process(request)
        except WorkerCrash:
            worker.kill()
            self._free_chain(rid)   # free before queueing: a crash leaks nothing
            self.safe_queue.append(request)
            return SAFE_QUEUE_PREFIX + request

    def drain_safe_queue(self) -> list[str]:
        drained = self.safe_queue[:]
        self.safe_queue.clear()
        results: list[str] = []
        for request in drained:
            try:
                results.append(self.submit(request))
            except RuntimeError:
                self.safe_queue.append(request)
                results.append(SAFE_QUEUE_PREFIX + request)
        return results

    # -- GPU data plane -------------------------------------------------------
    def admit(self, n_tokens: int, pool: int | None = None) -> int:
        """Registers a sequence with room for ``n_tokens`` and returns its id.

        Placement: the pool with the least resident tokens that has the
        blocks (or ``pool`` when given). The chain is allocated all-or-nothing.
        """
        if not self.pools:
            raise RuntimeError("this Supervisor owns no KV pools")
        if n_tokens < 0:
            raise RuntimeError(f"n_tokens must be >= 0, got {n_tokens}")
        nb = max(1, -(-n_tokens // BLOCK_SIZE))
        if pool is None:
            loads = self.pool_loads()
            ok = [p for p in range(len(self.pools)) if self.pools[p].table.num_free >= nb]
            if not ok:
                raise RuntimeError(f"insufficient free blocks: requested {nb} in any pool")
            pool = min(ok, key=lambda p: (loads[p], p))
        head = self.pools[pool].table.allocate_chain(nb)
        self._request_counter += 1
        rid = self._request_counter
        self.seqs[rid] = SeqState(pool=pool, head=head, length=0, blocks=nb)
        return rid

    def admit_many(self, lengths) -> list[int]:
        """Admits a batch with LPT placement over the pools (longest first)."""
        loads = self.pool_loads()
        where = lpt_placement(list(lengths), loads)
        return [self.admit(n, pool=p) for n, p in zip(lengths, where)]

    def pool_loads(self) -> list[int]:
        loads = [0] * len(self.pools)
        for st in self.seqs.values():
            loads[st.pool] += st.length
        return loads

    def reserve(self, rid: int, n_new: int) -> None:
        """Makes room for ``n_new`` more tokens, growing the chain at its tail."""
        st = self.seqs[rid]
        table = self.pools[st.pool].table
        have = table.chain_len(st.head) * BLOCK_SIZE
        need = st.length + n_new
        if need > have:
            tail = table.chain_tail(st.head)
            for _ in range(-(-(need - have) // BLOCK_SIZE)):
                tail = table.expand_chain(tail)
            st.blocks = table.chain_len(st.head)

    def finish(self, rid: int) -> None:
        """Frees a sequence's chain and forgets it."""
        st = self.seqs.pop(rid)
        self.pools[st.pool].table.free_chain(st.head)
        self._tables.clear()  # cached tables may name the freed chain

    def _device_table(self, p: int, rs):
        """Pool p's page table for ``rs`` on its device, kept between calls.

        The first call exports every row; later calls with the same sequences upload
        only the rows whose chain grew, and the whole table again only when the
        longest chain outgrows the kept width (kept in steps of 32 blocks).
        """
        import torch

        pool = self.pools[p]
        heads = tuple(self.seqs[r].head for r in rs)
        blocks = tuple(self.seqs[r].blocks for r in rs)
        need = max(blocks)
        key = (p, tuple(rs))
        ent = self._tables.get(key)
        if ent is None or ent["width"] < need or ent["heads"] != heads:
            width = -(-need // 32) * 32
            pt = pool.table.export_page_table(list(heads), width)
            if len(self._tables) >= 64:
                self._tables.clear()
            ent = {"width": width, "heads": heads, "blocks": blocks,
                   "pt": torch.from_numpy(pt).to(pool.device)}
            self._tables[key] = ent
        elif ent["blocks"] != blocks:
            rows = [i for i, (a, b) in enumerate(zip(ent["blocks"], blocks)) if a != b]
            fresh = pool.table.export_page_table([heads[i] for i in rows], ent["width"])
            idx = torch.tensor(rows, dtype=torch.long, device=pool.device)
            ent["pt"].index_copy_(0, idx, torch.from_numpy(fresh).to(pool.device))
            ent["blocks"] = blocks
        return ent["pt"], need

    def shard(self, rids) -> dict[int, tuple[list[int], object, object]]:
        """Per pool: (rids in order, page table [n, max_b] int32 numpy, lengths)."""
        import numpy as np

        by_pool: dict[int, list[int]] = {}
        for r in rids:
            by_pool.setdefault(self.seqs[r].pool, []).append(r)
        out = {}
        for p, rs in by_pool.items():
            table = self.pools[p].table
            heads = [self.seqs[r].head for r in rs]
            width = max(table.chain_len(h) for h in heads)
            pt = table.export_page_table(heads, width)
            lens = np.asarray([self.seqs[r].length for r in rs], dtype=np.int32)
            out[p] = (rs, pt, lens)
        return out

    def append_kv(self, rids, k_new, v_new, counts=None) -> None:
        """Writes new tokens' K/V ([n, Hkv, L, D] on the Supervisor device) into the pools.

        Chains are grown first; then each pool receives its rows and one
        kv-append kernel places them at positions length .. length + count - 1.
        """
        import torch

        from .kernels.block_attention import paged_kv_append

        L = k_new.shape[2]
        counts = [L] * len(rids) if counts is None else [int(c) for c in counts]
        for r, c in zip(rids, counts):
            self.reserve(r, c)
        index = {r: i for i, r in enumerate(rids)}
        for p, (rs, pt, _) in self.shard(rids).items():
            pool = self.pools[p]
            sel = torch.tensor([index[r] for r in rs], device=k_new.device)
            kp = k_new.index_select(0, sel).to(pool.device)
            vp = v_new.index_select(0, sel).to(pool.device)
            starts = torch.tensor([self.seqs[r].length for r in rs], dtype=torch.int32)
            cnt = torch.tensor([counts[index[r]] for r in rs], dtype=torch.int32)
            paged_kv_append(kp, vp, torch.from_numpy(pt), starts, cnt, pool.k_cache,
                            pool.v_cache)
        for r, c in zip(rids, counts):
            self.seqs[r].length += c

    def _gpu_worker(self, p: int) -> Worker:
        w = self._gpu_workers.get(p)
        if w is None or not w.alive:
            w = Worker(f"gpu{p}", device=self.pools[p].device)
            w.start()
            self._gpu_workers[p] = w
        return w

    def decode_step(self, rids, q, **kw):
        """Decode one token for each sequence in ``rids``.

        ``q`` is [len(rids), Hq, D] on the Supervisor's device. Each pool's
        shard runs on that pool's GPU through a stateless worker; outputs
        return to the Supervisor's device in ``rids`` order. A worker that
        crashes is replaced and its shard re-dispatched once; the KV pools
        are untouched by the crash because the Supervisor owns them.
        """
        import torch

        out = torch.empty_like(q)
        index = {r: i for i, r in enumerate(rids)}
        by_pool: dict[int, list[int]] = {}
        for r in rids:
            by_pool.setdefault(self.seqs[r].pool, []).append(r)
        pending = []
        for p, rs in by_pool.items():
            pool = self.pools[p]
            pt, _ = self._device_table(p, rs)
            lens = torch.tensor([self.seqs[r].length for r in rs], dtype=torch.int32)
            sel = torch.tensor([index[r] for r in rs], device=q.device)
            kw_p = dict(kw)
            nbs = [-(-self.seqs[r].length // BLOCK_SIZE) for r in rs]
            kw_p.setdefault("total_blocks", sum(nbs))
            kw_p.setdefault("max_seq_blocks", max(nbs))
            args = (pool.k_cache, pool.v_cache, pool.cos, pool.sin,
                    q.index_select(0, sel).to(pool.device), pt,
                    lens.to(pool.device, non_blocking=True))
            for attempt in range(2):
                worker = self._gpu_worker(p)
                try:
                    with torch.cuda.device(pool.device):
                        res = worker.decode(*args, **kw_p)
                    break
                except WorkerCrash:
                    worker.kill()
                    if attempt == 1:
                        raise
            pending.append((sel, res))
        for sel, res in pending:
            out.index_copy_(0, sel, res.to(q.device, non_blocking=True))
        return out


def pool_blocks_for(lengths, headroom: float = 0.05) -> int:
    """Blocks a pool needs for ``lengths`` tokens plus ``headroom``."""
    return int(math.ceil(sum(-(-n // BLOCK_SIZE) for n in lengths) * (1.0 + headroom))) + 1
