"""Continuous-batching serving loop: the Supervisor's per-GPU executor driving
the paged attention path end to end on a serving trace (Poisson arrivals,
lognormal prompt lengths, a fixed number of output tokens, token scopes from
random segments).

Per step, on one GPU's KV pool:

1. admission: arrived requests, in arrival order, get one chain for their
   prompt plus output tokens from the native allocator (all or nothing); a
   request that does not fit waits, and the queue behind it waits too;
2. prefill: up to ``prefill_tokens`` prompt tokens, at most ``chunk`` per
   request: stand-in QKV projection, the chunk's K/V appended to the chain
   (kv-append kernel), causal attention of the chunk over the chain under
   the request's token scope (tensor-core prefill kernel); a request whose
   prompt completes gets its first output token from the prompt's last row;
3. decode: every request past its prompt decodes one token: QKV projection of
   its last token, K/V append, paged decode attention under the request's
   token scope (decode kernel), output projection, next token;
4. a request with all its output tokens frees its chain.

The model around attention is a random-init stand-in (token embedding, fused
QKV projection, output projection and an argmax over the first ``vocab``
hidden units as the next token): the trace exercises the allocator and the
attention kernels, not a language model.

The scheduler talks to a backend (``admit`` / ``prefill`` / ``decode`` /
``release``), so it runs on the CPU against a stand-in backend in the tests.
It needs token counts, never token values, and hands the backend each chain
once, at admission: the GPU backend keeps page-table rows, scopes and last
tokens resident per slot, so a step costs one small host-to-device copy of
its indices and no page-table rebuild.
"""

from __future__ import annotations

import math
import random
import time
from collections import deque
from dataclasses import dataclass, field

import numpy as np

from .block_table import BLOCK_SIZE
from .scoping_mask import GLOBAL, LOCAL, token_scope


@dataclass
class Request:
    rid: int
    arrival: float          # seconds after the trace starts
    prompt_len: int
    max_new: int            # output tokens (the first comes from the prefill)
    spans: list             # [(start, end, scope)] partitioning [0, prompt_len + max_new)
    head: int = -1          # chain head while admitted
    slot: int = -1          # backend slot while admitted
    done_prompt: int = 0    # prompt tokens whose K/V are in the cache
    generated: int = 0      # output tokens produced
    last_token: int = 0
    admit_time: float | None = None
    first_token_time: float | None = None
    finish_time: float | None = None
    first_token_step: int | None = None  # the step that produced the first token
    finish_step: int | None = None       # the step that produced the last one
    tags: np.ndarray | None = field(default=None, repr=False)   # uint8 [total], 1 = GLOBAL
    span_start: np.ndarray | None = field(default=None, repr=False)
    span_end: np.ndarray | None = field(default=None, repr=False)

    @property
    def total(self) -> int:
        return self.prompt_len + self.max_new

    @property
    def blocks(self) -> int:
        return -(-self.total // BLOCK_SIZE)

    def scope_span(self, pos: int) -> tuple[int, int]:
        """(lo, hi) of the query at ``pos``: empty for a GLOBAL query."""
        if self.tags[pos]:
            return 0, 0
        return int(self.span_start[pos]), int(self.span_end[pos])


def random_segments(rng: random.Random, total: int, lo: int = 32, hi: int = 512) -> list:
    """Segments of U[lo, hi] tokens covering [0, total) (the last one truncated):
    the first GLOBAL, each later one LOCAL with probability 1/2, else GLOBAL."""
    spans, s, k = [], 0, 0
    while s < total:
        e = min(total, s + rng.randint(lo, hi))
        spans.append((s, e, GLOBAL if k == 0 or rng.random() >= 0.5 else LOCAL))
        s, k = e, k + 1
    return spans


def make_trace(n: int, rate: float, median: float, sigma: float, lo: int, hi: int,
               max_new: int, seed: int) -> list[Request]:
    """Poisson arrivals at ``rate`` per second, prompt lengths lognormal with the
    given median and sigma clipped to [lo, hi], ``max_new`` output tokens."""
    rng = random.Random(seed)
    t, out = 0.0, []
    for i in range(n):
        t += rng.expovariate(rate)
        L = int(min(hi, max(lo, round(rng.lognormvariate(math.log(median), sigma)))))
        out.append(Request(i, t, L, max_new, random_segments(rng, L + max_new)))
    return out


class Engine:
    """Continuous batching over one pool's allocator (``table``) and a backend."""

    def __init__(self, table, backend, *, chunk: int = 2048, prefill_tokens: int = 8192,
                 slots: int = 1024):
        self.table = table
        self.backend = backend
        self.chunk = chunk
        self.prefill_tokens = prefill_tokens
        self.waiting: deque[Request] = deque()
        self.running: list[Request] = []
        self.finished: list[Request] = []
        self.free_slots = list(range(slots - 1, -1, -1))
        self.steps = 0
        self.peak_running = 0
        self.peak_blocks = 0

    def submit(self, reqs) -> None:
        self.waiting.extend(sorted(reqs, key=lambda r: (r.arrival, r.rid)))

    @property
    def idle(self) -> bool:
        return not self.waiting and not self.running

    def _admit(self, now: float) -> None:
        while self.waiting and self.waiting[0].arrival <= now and self.free_slots:
            r = self.waiting[0]
            if self.table.num_free < r.blocks:
                break                       # arrival order: the queue waits behind r
            r.head = self.table.allocate_chain(r.blocks)
            r.slot = self.free_slots.pop()
            r.tags, r.span_start, r.span_end = token_scope(r.spans)
            r.admit_time = now
            self.backend.admit(r, list(self.table.walk(r.head)))
            self.running.append(r)
            self.waiting.popleft()

    def page_table(self, reqs):
        """Host page table of ``reqs`` (one native export; the GPU backend keeps its own)."""
        width = max(self.table.chain_len(r.head) for r in reqs)
        return self.table.export_page_table([r.head for r in reqs], width)

    def step(self, now: float) -> None:
        """One scheduling step at time ``now``; a no-op when nothing is runnable."""
        self._admit(now)
        # prefill: oldest prompts first, at most `chunk` tokens each, `prefill_tokens` in all
        pre, starts, counts, budget = [], [], [], self.prefill_tokens
        for r in self.running:
            left = r.prompt_len - r.done_prompt
            if left > 0 and budget > 0:
                c = min(left, self.chunk, budget)
                pre.append(r)
                starts.append(r.done_prompt)
                counts.append(c)
                budget -= c
        dec = [r for r in self.running if r.done_prompt == r.prompt_len and 0 < r.generated < r.max_new]
        if pre:
            tokens = self.backend.prefill(pre, np.asarray(starts, np.int32),
                                          np.asarray(counts, np.int32))
            for i, (r, c) in enumerate(zip(pre, counts)):
                r.done_prompt += c
                if r.done_prompt == r.prompt_len:
                    if tokens is not None:
                        r.last_token = int(tokens[i])
                    r.generated = 1
                    r.first_token_time = now
                    r.first_token_step = self.steps
        if dec:
            pos = np.asarray([r.prompt_len + r.generated - 1 for r in dec], np.int32)
            tokens = self.backend.decode(dec, pos)
            for i, r in enumerate(dec):
                if tokens is not None:
                    r.last_token = int(tokens[i])
                r.generated += 1
        if pre or dec:
            self.steps += 1
        self.peak_running = max(self.peak_running, len(self.running))
        self.peak_blocks = max(self.peak_blocks, self.table.max_blocks - self.table.num_free)
        keep = []
        for r in self.running:
            if r.generated >= r.max_new:
                if r.first_token_time is None:
                    r.first_token_time = now
                    r.first_token_step = self.steps - 1
                r.finish_time = now
                r.finish_step = self.steps - 1
                self.table.free_chain(r.head)
                self.backend.release(r)
                self.free_slots.append(r.slot)
                r.head = r.slot = -1
                self.finished.append(r)
            else:
                keep.append(r)
        self.running = keep

    def run(self, reqs, *, clock=time.perf_counter, sleep=time.sleep, sync=None,
            timer=None, max_steps: int = 10 ** 9) -> dict:
        """Serves ``reqs`` with arrivals on ``clock`` (seconds since the call) and
        returns the trace's statistics. ``sync`` (optional) waits for the device
        after every step, so host timestamps follow the device. ``timer``
        (optional, instead) keeps the host free to run ahead: ``timer.start()``
        at the start, ``timer.mark()`` after every step that did work (a device
        marker, e.g. a CUDA event), ``timer.sync()`` once at the end and
        ``timer.seconds(marker)`` since the start; first-token and finish times
        are then those of the steps that produced the tokens."""
        self.submit(reqs)
        marks = []
        if timer is not None:
            timer.start()
        t0 = clock()
        while not self.idle and self.steps < max_steps:
            now = clock() - t0
            if not self.running and self.waiting and self.waiting[0].arrival > now:
                sleep(min(0.001, self.waiting[0].arrival - now))
                continue
            before = self.steps
            self.step(now)
            if timer is not None and self.steps > before:
                marks.append(timer.mark())
            if sync is not None:
                sync()
        if timer is not None:
            timer.sync()
            for r in self.finished:
                if r.first_token_step is not None:
                    r.first_token_time = timer.seconds(marks[r.first_token_step])
                if r.finish_step is not None:
                    r.finish_time = timer.seconds(marks[r.finish_step])
        wall = clock() - t0
        return self.stats(wall)

    def stats(self, wall: float) -> dict:
        done = self.finished
        gen = sum(r.generated for r in done)
        ttft = [r.first_token_time - r.arrival for r in done if r.first_token_time is not None]
        tpot = [(r.finish_time - r.first_token_time) / (r.max_new - 1)
                for r in done if r.max_new > 1 and r.first_token_time is not None]
        q = lambda xs, p: float(np.percentile(xs, p)) if xs else None  # noqa: E731
        return {
            "requests": len(done), "generated_tokens": gen, "wall_s": wall, "steps": self.steps,
            "prompt_tokens": sum(r.prompt_len for r in done),
            "ttft_s": {"p50": q(ttft, 50), "p99": q(ttft, 99)},
            "tpot_s": {"p50": q(tpot, 50), "p99": q(tpot, 99)},
            "peak_running": self.peak_running, "peak_blocks": self.peak_blocks,
        }


def shard_requests(reqs, world: int) -> list[list[Request]]:
    """Whole requests per GPU, longest-processing-time on total tokens (the
    Supervisor's placement), in arrival order within each shard."""
    loads = [0] * world
    out = [[] for _ in range(world)]
    for r in sorted(reqs, key=lambda r: (-r.total, r.rid)):
        g = min(range(world), key=lambda i: (loads[i], i))
        loads[g] += r.total
        out[g].append(r)
    return [sorted(s, key=lambda r: (r.arrival, r.rid)) for s in out]


class StandInBackend:
    """Random-init stand-in model on one GPU around the paged attention path.

    Weights (bf16, N(0, 1/hidden)): token embedding [vocab, hidden], fused QKV
    projection [hidden, (Hq + 2 Hkv) D], output projection [Hq D, hidden]. A
    prompt token's id is a fixed hash of (request, position); the next token
    is the argmax over the first ``vocab`` units of the projected attention
    output. Per slot, on the device: the chain's page-table row (written at
    admission, PAD past it), the token scope (tags and per-position spans)
    and the last token. A step uploads its indices once (pinned buffer,
    asynchronous copy) and reads nothing back. ``kv_bytes`` counts the cached
    bytes decode attention covers and ``attn_ms`` the attention launches'
    device time (CUDA events on the launching stream).
    """

    def __init__(self, pool, q_heads: int, *, hidden: int = 4096, vocab: int = 4096,
                 max_total: int = 16640, slots: int = 1024, seed: int = 0):
        import torch

        self.torch = torch
        self.pool = pool
        self.device = pool.device
        self.hq, self.hkv, self.d = q_heads, pool.kv_heads, pool.head_dim
        self.vocab = vocab
        g = torch.Generator(device=self.device).manual_seed(seed)
        dt = pool.dtype
        scale = 1.0 / math.sqrt(hidden)
        self.emb = (torch.randn(vocab, hidden, generator=g, device=self.device)).to(dt)
        self.w_qkv = (torch.randn(hidden, (self.hq + 2 * self.hkv) * self.d, generator=g,
                                  device=self.device) * scale).to(dt)
        self.w_o = (torch.randn(self.hq * self.d, hidden, generator=g, device=self.device)
                    * (1.0 / math.sqrt(self.hq * self.d))).to(dt)
        width = -(-max_total // 16) * 16
        self.max_blocks = -(-max_total // BLOCK_SIZE)
        dev = self.device
        # per-slot state: page-table row, token scope (GLOBAL tags, span of the token at each
        # position), last token
        self.pt = torch.full((slots, self.max_blocks), -1, dtype=torch.int32, device=dev)
        self.tags = torch.zeros(slots, width, dtype=torch.uint8, device=dev)
        self.span_lo = torch.zeros(slots, width, dtype=torch.int32, device=dev)
        self.span_hi = torch.zeros(slots, width, dtype=torch.int32, device=dev)
        self.last_tok = torch.zeros(slots, dtype=torch.int64, device=dev)
        # per-step indices: two pinned staging buffers, each reused once the copy that
        # last read it has completed
        self._stage = [torch.empty(8 * slots, dtype=torch.int32, pin_memory=True) for _ in range(2)]
        self._stage_done = [None, None]
        self._flip = 0
        # decode inputs gathered per step into fixed buffers, and one prepared decode call per
        # batch size over their first n rows (checks, plan and workspace done once per size)
        self._dec = {"pt": torch.full((slots, self.max_blocks), -1, dtype=torch.int32, device=dev),
                     "q": torch.empty(slots, self.hq, self.d, dtype=dt, device=dev),
                     "lens": torch.zeros(slots, dtype=torch.int32, device=dev),
                     "tags": torch.zeros(slots, width, dtype=torch.uint8, device=dev),
                     "span": torch.zeros(slots, 2, dtype=torch.int32, device=dev)}
        self._dec_calls = {}
        self.kv_bytes = 0
        self.attn_events = {"prefill": [], "decode": []}  # (start, end) CUDA event pairs
        self.last_prefill = self.last_decode = None        # inputs / outputs of the last call

    # ---- slots ------------------------------------------------------------
    def admit(self, r: Request, blocks) -> None:
        torch = self.torch
        row = torch.full((self.max_blocks,), -1, dtype=torch.int32)
        row[: len(blocks)] = torch.tensor(blocks, dtype=torch.int32)
        self.pt[r.slot].copy_(row)
        self.tags[r.slot].zero_()
        self.tags[r.slot, : r.total].copy_(torch.from_numpy(r.tags))
        self.span_lo[r.slot, : r.total].copy_(torch.from_numpy(r.span_start))
        self.span_hi[r.slot, : r.total].copy_(torch.from_numpy(r.span_end))

    def release(self, r: Request) -> None:
        pass

    def _upload(self, cols):
        """int32 host columns of equal length -> device [len(cols), n] in one async copy."""
        torch = self.torch
        n = len(cols[0])
        buf = self._stage[self._flip]
        if self._stage_done[self._flip] is not None:
            self._stage_done[self._flip].synchronize()
        host = buf[: len(cols) * n].view(len(cols), n)
        for i, c in enumerate(cols):
            host[i].copy_(torch.from_numpy(np.ascontiguousarray(c, dtype=np.int32)))
        dev = host.to(self.device, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self._stage_done[self._flip] = ev
        self._flip ^= 1
        return dev

    # ---- model pieces -------------------------------------------------------
    def _qkv(self, tokens):
        """tokens [...] int64 -> q [..., Hq, D], k / v [..., Hkv, D]."""
        h = self.emb[tokens]
        qkv = (h @ self.w_qkv).view(*tokens.shape, self.hq + 2 * self.hkv, self.d)
        return qkv[..., : self.hq, :], qkv[..., self.hq: self.hq + self.hkv, :], qkv[..., self.hq + self.hkv:, :]

    def _next(self, o):
        """o [n, Hq, D] -> next token ids [n] (device)."""
        h = o.reshape(o.shape[0], -1) @ self.w_o
        return h[:, : self.vocab].float().argmax(dim=1)

    def _timed(self, kind, fn):
        torch = self.torch
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        out = fn()
        e1.record()
        self.attn_events[kind].append((e0, e1))
        return out

    def attn_ms(self, kind=None) -> float:
        """Device time of the attention launches (``"prefill"``, ``"decode"`` or both)."""
        self.torch.cuda.synchronize(self.device)
        kinds = [kind] if kind else list(self.attn_events)
        return sum(a.elapsed_time(b) for k in kinds for a, b in self.attn_events[k])

    # ---- backend interface ---------------------------------------------------
    def prefill(self, reqs, starts, counts):
        from .kernels.block_attention import chunked_prefill_attention, paged_kv_append

        torch = self.torch
        dev = self.device
        n, Lc = len(reqs), int(counts.max())
        done = np.asarray([s + c == r.prompt_len for r, s, c in zip(reqs, starts, counts)], np.int32)
        idx = self._upload([[r.slot for r in reqs], [r.rid for r in reqs], starts, counts, done])
        slots, rids, st, ct, fin = idx[0], idx[1], idx[2], idx[3], idx[4]
        pos = st[:, None].long() + torch.arange(Lc, device=dev)[None, :]
        tokens = (rids[:, None].long() * 7919 + pos * 104729) % self.vocab
        q, k, v = self._qkv(tokens)                          # [n, Lc, H, D]
        q = q.permute(0, 2, 1, 3).contiguous()
        k = k.permute(0, 2, 1, 3).contiguous()
        v = v.permute(0, 2, 1, 3).contiguous()
        pt = self.pt.index_select(0, slots)
        paged_kv_append(k, v, pt, st, ct, self.pool.k_cache, self.pool.v_cache)
        scope = (self.tags.index_select(0, slots), self.span_lo.index_select(0, slots),
                 self.span_hi.index_select(0, slots))
        out = self._timed("prefill", lambda: chunked_prefill_attention(
            pt, q, self.pool.k_cache, self.pool.v_cache, st, st + ct, self.pool.cos,
            self.pool.sin, causal=True, validate=False, scope=scope))
        self.last_prefill = (pt, q, st, st + ct, scope, out)
        last = out[torch.arange(n, device=dev), :, ct.long() - 1]   # [n, Hq, D]
        nxt = self._next(last)
        # requests whose prompt is complete take their first output token
        self.last_tok.index_copy_(0, slots.long(),
                                  torch.where(fin != 0, nxt, self.last_tok.index_select(0, slots)))
        return None

    def _decode_call(self, n):
        """The prepared decode launch over the first m >= n rows of the decode buffers, m
        rounded up to a multiple of 8 (rows n .. m - 1 get length 0: no keys, zero output),
        so a run keeps at most slots / 8 prepared calls."""
        m = min(-(-n // 8) * 8, self._dec["lens"].shape[0])
        if m > n:
            self._dec["lens"][n:m].zero_()
        call = self._dec_calls.get(m)
        if call is None:
            from .kernels.block_attention import DecodeCall

            b = self._dec
            call = DecodeCall(b["pt"][:m], b["q"][:m], self.pool.k_cache, self.pool.v_cache,
                              b["lens"][:m], self.pool.cos, self.pool.sin,
                              scope=(b["tags"][:m], b["span"][:m]), validate=False)
            self._dec_calls[m] = call
        return call

    def decode(self, reqs, pos):
        from .kernels.block_attention import paged_kv_append

        torch = self.torch
        dev = self.device
        n = len(reqs)
        spans = [r.scope_span(int(p)) for r, p in zip(reqs, pos)]
        idx = self._upload([[r.slot for r in reqs], pos, [a for a, _ in spans],
                            [b for _, b in spans]])
        slots, start = idx[0], idx[1]
        b = self._dec
        pt, lens, tags, span = b["pt"][:n], b["lens"][:n], b["tags"][:n], b["span"][:n]
        torch.index_select(self.pt, 0, slots, out=pt)
        torch.index_select(self.tags, 0, slots, out=tags)
        span.copy_(idx[2:4].t())
        torch.add(start, 1, out=lens)
        q, k, v = self._qkv(self.last_tok.index_select(0, slots))   # [n, H, D]
        b["q"][:n].copy_(q)
        q = b["q"][:n]
        paged_kv_append(k[:, :, None].contiguous(), v[:, :, None].contiguous(), pt, start,
                        torch.ones(n, dtype=torch.int32, device=dev), self.pool.k_cache,
                        self.pool.v_cache)
        call = self._decode_call(n)
        out = self._timed("decode", call.launch)[:n]
        self.kv_bytes += int(pos.astype(np.int64).sum() + n) * self.hkv * self.d * 2 * \
            self.pool.k_cache.element_size()
        self.last_decode = (pt, q, lens, tags, span, out)
        self.last_tok.index_copy_(0, slots.long(), self._next(out))
        return None
