"""Multi-process plumbing for the sharded decode step (one process per GPU).

Rank 0 hosts the Supervisor: it holds every pool's allocator and builds each
rank's page-table slice; each rank's process owns its GPU's caches and runs a
stateless worker. Per step:

  1. rank 0 scatters the query shards and page-table slices (padded to the
     largest shard so every rank receives equal-sized tensors);
  2. every rank runs its shard;
  3. rank 0 gathers the outputs (NCCL over NVLink on B200; gloo on CPU) and
     drops the padding.

Every rank takes the same collective calls in the same order on every path.
The compute of step 2 is a function argument, so the routing is testable on
CPU ranks with gloo.

:func:`sharded_step` is the one-shot form (shapes travel in a header every
call); :class:`DecodeShards` is the repeated form for a fixed batch: shapes
and buffers are fixed once, and a step is one permute, one point-to-point
group out, the decode, one group back and one permute.
"""

from __future__ import annotations

from typing import Callable


def padded_shards(shards: list, width: int, pad_value=0):
    """Pads each [n_r, ...] shard to [width, ...] along dim 0."""
    import torch

    out = []
    for t in shards:
        if t.shape[0] > width:
            raise RuntimeError("shard larger than the scatter width")
        pad = torch.full((width - t.shape[0],) + tuple(t.shape[1:]), pad_value, dtype=t.dtype,
                         device=t.device)
        out.append(torch.cat([t, pad], dim=0))
    return out


def sharded_step(compute: Callable, world: int, rank: int, device, *, q_shards=None,
                 pt_shards=None, len_shards=None, q_shape=None, pt_width=None, group=None):
    """One scatter -> compute -> gather round; returns the gathered rows on rank 0.

    On rank 0 ``q_shards``/``pt_shards``/``len_shards`` hold one tensor per rank
    ([n_r, Hq, D], [n_r, W_r] int32, [n_r] int32). Other ranks pass None and
    the broadcast header tells them the padded shapes. ``compute(q, pt, lens)``
    runs on every rank and returns [n, Hq, D]. Rank 0 gets a list of per-rank
    outputs with padding removed; other ranks get None.
    """
    import torch
    import torch.distributed as dist

    hdr = torch.zeros(world + 4, dtype=torch.int64, device=device)
    if rank == 0:
        width = max(t.shape[0] for t in q_shards)
        ptw = max(t.shape[1] for t in pt_shards)
        hdr[0], hdr[1], hdr[2], hdr[3] = width, ptw, q_shards[0].shape[1], q_shards[0].shape[2]
        for r in range(world):
            hdr[4 + r] = q_shards[r].shape[0]
    dist.broadcast(hdr, src=0, group=group)
    width, ptw, hq, d = (int(x) for x in hdr[:4].tolist())
    counts = [int(x) for x in hdr[4:].tolist()]
    qdtype = q_shards[0].dtype if rank == 0 else None
    dt = torch.zeros(1, dtype=torch.int64, device=device)
    if rank == 0:
        dt[0] = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[qdtype]
    dist.broadcast(dt, src=0, group=group)
    qdtype = (torch.float32, torch.float16, torch.bfloat16)[int(dt.item())]

    q_recv = torch.empty((width, hq, d), dtype=qdtype, device=device)
    pt_recv = torch.empty((width, ptw), dtype=torch.int32, device=device)
    len_recv = torch.empty((width,), dtype=torch.int32, device=device)
    if rank == 0:
        qs = padded_shards(q_shards, width)
        pts = padded_shards([torch.nn.functional.pad(t, (0, ptw - t.shape[1]), value=-1)
                             for t in pt_shards], width, pad_value=-1)
        ls = padded_shards(len_shards, width)
    else:
        qs = pts = ls = None
    dist.scatter(q_recv, qs, src=0, group=group)
    dist.scatter(pt_recv, pts, src=0, group=group)
    dist.scatter(len_recv, ls, src=0, group=group)
    mine = counts[rank]
    out = compute(q_recv[:mine], pt_recv[:mine], len_recv[:mine])
    out_full = torch.zeros((width, hq, d), dtype=qdtype, device=device)
    out_full[:mine] = out
    gathered = [torch.empty_like(out_full) for _ in range(world)] if rank == 0 else None
    dist.gather(out_full, gathered, dst=0, group=group)
    if rank != 0:
        return None
    return [g[:c] for g, c in zip(gathered, counts)]


class _DevBytes:
    """A device address range as a CUDA-array-interface object (zero-copy torch view)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                         "data": (ptr, False), "version": 3}


def _view(torch, ptr: int, shape, dtype, device):
    """A torch tensor over device memory at ``ptr`` (not owned by torch)."""
    n = 1
    for x in shape:
        n *= int(x)
    nbytes = n * torch.tensor([], dtype=dtype).element_size()
    if nbytes == 0:
        return torch.empty(shape, dtype=dtype, device=device)
    raw = torch.as_tensor(_DevBytes(ptr, nbytes), device=device)
    if raw.data_ptr() != ptr:
        raise RuntimeError("could not view the shared buffer without a copy")
    return raw.view(dtype).view(shape)


def _align(x: int, a: int = 256) -> int:
    return -(-x // a) * a


class DecodeShards:
    """Repeated sharded decode of one batch over one process per GPU.

    Rank 0 hosts the Supervisor. It owns every pool's allocator, holds the
    batch's queries in batch order, and fixes at set-up which rank holds which
    sequences (``placement``, e.g. longest-processing-time placement by token
    count, :func:`src.serving.lpt_placement`). Set-up is collective and runs
    once per batch composition: one broadcast tells every rank its shard size
    and page-table width, and every buffer is allocated then. A step is
    collective too and does no host work beyond enqueueing:

      1. rank 0 permutes the queries into shard order;
      2. each rank r > 0 gets its query rows and its metadata (the shard's
         lengths followed by its page-table rows, one int32 buffer); rank 0's
         own shard is read in place;
      3. every rank runs ``run()``, which must decode ``q`` / ``page_table`` /
         ``seq_lens`` into the rows at ``out_ptr`` (``out`` is their tensor, None
         on a worker of the peer exchange, whose rows live in rank 0's buffer);
      4. rank 0 gets every shard's output rows and restores the batch order.

    Two exchanges. ``exchange="nccl"`` moves steps 2 and 4 as NCCL
    point-to-point groups (any backend: gloo on CPU ranks). ``exchange="peer"``
    (CUDA, one GPU per rank) shares buffers through CUDA IPC and moves them with
    the library's kernels: rank 0's permute writes the rows into its shared
    buffer and raises every worker's ready flag; a worker's fetch kernel waits
    for its flag and copies its rows and metadata over NVLink; the worker's
    decode writes its output rows straight into rank 0's shared buffer, its
    signal kernel raises its done flag there, and rank 0's collect kernel waits
    for every flag and restores the batch order. Every wait is bounded
    (``timeout_s``; status bit 2 in ``exchange_status`` when it runs out).

    Every rank calls the same collectives in the same order; every rank must
    hold at least one sequence. The metadata is resent every step because the
    lengths grow by one token per step and a chain gains a block every 64
    tokens; ``set_meta`` (rank 0) rewrites it. ``close()`` (collective) releases
    the shared buffers.
    """

    def __init__(self, world: int, rank: int, device, *, q_heads: int, head_dim: int, dtype,
                 placement=None, widths=None, group=None, exchange: str = "nccl",
                 timeout_s: float = 2.0):
        import torch
        import torch.distributed as dist

        if exchange not in ("nccl", "peer"):
            raise RuntimeError(f"exchange must be 'nccl' or 'peer', got {exchange!r}")
        self.world, self.rank, self.device, self.group = world, rank, device, group
        self.exchange = exchange if world > 1 else "nccl"
        self.timeout_ns = int(timeout_s * 1e9)
        self.step_no = 0
        hdr = torch.zeros(2 * world, dtype=torch.int64, device=device)
        if rank == 0:
            if placement is None or widths is None or len(widths) != world:
                raise RuntimeError("rank 0 needs the placement and one page-table width per rank")
            counts = [0] * world
            for r in placement:
                if not 0 <= int(r) < world:
                    raise RuntimeError(f"placement names rank {r} outside [0, {world})")
                counts[int(r)] += 1
            hdr[:world] = torch.tensor(counts, dtype=torch.int64)
            hdr[world:] = torch.tensor([int(w) for w in widths], dtype=torch.int64)
        if world > 1:
            dist.broadcast(hdr, src=0, group=group)
        vals = [int(x) for x in hdr.tolist()]
        self.counts, self.widths = vals[:world], vals[world:]
        if min(self.counts) < 1:
            raise RuntimeError(f"every rank must hold a sequence, shard sizes {self.counts}")
        if min(self.widths) < 1:
            raise RuntimeError(f"page-table widths must be >= 1, got {self.widths}")
        self.n, self.width = self.counts[rank], self.widths[rank]
        self.q_off = [sum(self.counts[:r]) for r in range(world)]
        # metadata segments padded to 16 bytes (four int32)
        self.meta_len = [_align(c * (1 + w), 4) for c, w in zip(self.counts, self.widths)]
        self.meta_off = [sum(self.meta_len[:r]) for r in range(world)]
        S = sum(self.counts)
        self.S = S
        qshape = (q_heads, head_dim)
        self.row_bytes = q_heads * head_dim * torch.tensor([], dtype=dtype).element_size()
        if rank == 0:
            order = sorted(range(S), key=lambda i: (int(placement[i]), i))
            self.batch_index = order  # shard-order position -> batch index
            self.perm = torch.tensor(order, dtype=torch.int64, device=device)
            inv = [0] * S
            for pos, i in enumerate(order):
                inv[i] = pos
            self.inv = torch.tensor(inv, dtype=torch.int64, device=device)
            self.out_batch = torch.empty((S,) + qshape, dtype=dtype, device=device)
        self.exchange_status = torch.zeros(1, dtype=torch.int32, device=device)
        self._own = self._p0 = None
        self._peers = []
        if self.exchange == "peer":
            self._setup_peer(torch, dist, qshape, dtype)
        elif rank == 0:
            self.q_perm = torch.empty((S,) + qshape, dtype=dtype, device=device)
            self.meta_all = torch.zeros(sum(self.meta_len), dtype=torch.int32, device=device)
            self.out_perm = torch.empty((S,) + qshape, dtype=dtype, device=device)
        else:
            self.q = torch.empty((self.n,) + qshape, dtype=dtype, device=device)
            self.meta = torch.zeros(self.meta_len[rank], dtype=torch.int32, device=device)
            self.out = torch.empty((self.n,) + qshape, dtype=dtype, device=device)
        if rank == 0:
            self.q = self.q_perm[:self.n]
            self.meta = self.meta_all[:self.meta_len[0]]
            self.out = self.out_perm[:self.n]
        if self.out is not None:
            self.out_ptr = self.out.data_ptr()
        self.seq_lens = self.meta[:self.n]
        self.page_table = self.meta[self.n:self.n * (1 + self.width)].view(self.n, self.width)

    # -- the peer-memory exchange -------------------------------------------------------
    def _layout(self):
        """Byte offsets of rank 0's shared buffer: flags, queries, metadata, outputs."""
        flags = _align(64 * (self.world + 1))
        q = flags
        meta = _align(q + self.S * self.row_bytes)
        out = _align(meta + sum(self.meta_len) * 4)
        return flags, q, meta, out, _align(out + self.S * self.row_bytes)

    def _setup_peer(self, torch, dist, qshape, dtype):
        import ctypes

        from . import _native
        from .kernels import _capi  # noqa: F401  (registers the exchange symbols)

        lib = _native.lib()
        flags, q_b, meta_b, out_b, total = self._layout()
        own = ctypes.c_void_p()
        _native.check(lib.ouro_ipc_alloc(total if self.rank == 0 else flags, ctypes.byref(own)),
                      "ipc alloc")
        self._own = own.value
        h = (ctypes.c_uint8 * 64)()
        _native.check(lib.ouro_ipc_handle(self._own, h), "ipc handle")
        mine = torch.tensor(list(bytes(h)), dtype=torch.uint8, device=self.device)
        handles = [torch.empty_like(mine) for _ in range(self.world)]
        dist.all_gather(handles, mine, group=self.group)
        handles = [bytes(x.cpu().tolist()) for x in handles]
        dev = self.device
        if self.rank == 0:
            for r in range(1, self.world):
                p = ctypes.c_void_p()
                buf = (ctypes.c_uint8 * 64).from_buffer_copy(handles[r])
                _native.check(lib.ouro_ipc_open(buf, ctypes.byref(p)), "ipc open")
                self._peers.append(p.value)
            # each worker's ready flag is the first word of its shared buffer
            self._ready_ptrs = torch.tensor(self._peers, dtype=torch.int64, device=dev)
            self.q_perm = _view(torch, self._own + q_b, (self.S,) + qshape, dtype, dev)
            self.meta_all = _view(torch, self._own + meta_b, (sum(self.meta_len),), torch.int32,
                                  dev)
            self.out_perm = _view(torch, self._own + out_b, (self.S,) + qshape, dtype, dev)
        else:
            p = ctypes.c_void_p()
            buf = (ctypes.c_uint8 * 64).from_buffer_copy(handles[0])
            _native.check(lib.ouro_ipc_open(buf, ctypes.byref(p)), "ipc open")
            self._p0 = p.value
            r = self.rank
            self.q = torch.empty((self.n,) + qshape, dtype=dtype, device=dev)
            self.meta = torch.zeros(self.meta_len[r], dtype=torch.int32, device=dev)
            # the decode writes this rank's rows straight into rank 0's buffer: a raw
            # address (out_ptr), since the memory belongs to rank 0's GPU
            self.out = None
            self.out_ptr = self._p0 + out_b + self.q_off[r] * self.row_bytes
            self._src_q = self._p0 + q_b + self.q_off[r] * self.row_bytes
            self._src_meta = self._p0 + meta_b + self.meta_off[r] * 4
            self._done_flag = self._p0 + 64 * r
        torch.cuda.synchronize(dev)
        dist.barrier(group=self.group)

    def close(self) -> None:
        """Collective: unmaps the peers' buffers, then frees this rank's shared buffer."""
        if self.exchange != "peer" or self._own is None:
            return
        import torch
        import torch.distributed as dist

        from . import _native

        lib = _native.lib()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for ptr in self._peers + ([self._p0] if self._p0 else []):
            _native.check(lib.ouro_ipc_close(ptr), "ipc close")
        self._peers, self._p0 = [], None
        dist.barrier(group=self.group)
        _native.check(lib.ouro_ipc_free(self._own), "ipc free")
        self._own = None
        for name in ("q_perm", "meta_all", "out_perm", "q", "meta", "out", "seq_lens",
                     "page_table"):
            if hasattr(self, name):
                setattr(self, name, None)

    def _stream(self):
        import torch

        return torch.cuda.current_stream(self.device).cuda_stream

    def shard_of(self, r: int) -> list[int]:
        """Rank 0: the batch indices rank r holds, in its shard order."""
        return self.batch_index[self.q_off[r]:self.q_off[r] + self.counts[r]]

    def set_meta(self, lens_per_rank, pt_per_rank) -> None:
        """Rank 0: writes every shard's lengths [n_r] and page-table rows [n_r, w_r]."""
        import torch

        if self.rank != 0:
            raise RuntimeError("set_meta runs on the Supervisor's rank (0)")
        for r in range(self.world):
            ln = torch.as_tensor(lens_per_rank[r], dtype=torch.int32).reshape(-1)
            pt = torch.as_tensor(pt_per_rank[r], dtype=torch.int32)
            if ln.numel() != self.counts[r] or tuple(pt.shape) != (self.counts[r], self.widths[r]):
                raise RuntimeError(f"rank {r}: lengths / page table do not match the shard "
                                   f"({self.counts[r]} sequences, width {self.widths[r]})")
            c = self.counts[r]
            seg = self.meta_all[self.meta_off[r]:self.meta_off[r] + self.meta_len[r]]
            seg[:c].copy_(ln, non_blocking=True)
            seg[c:c * (1 + self.widths[r])].copy_(pt.reshape(-1), non_blocking=True)

    def _exchange(self, ops) -> None:
        import torch.distributed as dist

        if ops:
            for w in dist.batch_isend_irecv(ops):
                w.wait()

    def scatter(self, q_batch=None) -> None:
        """Step parts 1-2: rank 0 passes the batch's queries [S, Hq, D]."""
        import torch
        import torch.distributed as dist

        self.step_no += 1
        if self.exchange == "peer":
            from . import _native

            lib = _native.lib()
            if self.rank == 0:
                q_batch = q_batch.contiguous()
                _native.check(lib.ouro_shard_publish(
                    q_batch.data_ptr(), self.perm.data_ptr(), self.q_perm.data_ptr(), self.S,
                    self.row_bytes, self._ready_ptrs.data_ptr(), self.world - 1, self.step_no,
                    self._stream()), "shard publish")
            else:
                _native.check(lib.ouro_shard_fetch(
                    self._own, self.step_no, self.timeout_ns, self._src_q, self.q.data_ptr(),
                    self.n * self.row_bytes, self._src_meta, self.meta.data_ptr(),
                    self.meta_len[self.rank] * 4, self.exchange_status.data_ptr(),
                    self._stream()), "shard fetch")
            return
        ops = []
        if self.rank == 0:
            torch.index_select(q_batch, 0, self.perm, out=self.q_perm)
            for r in range(1, self.world):
                ops.append(dist.P2POp(dist.isend, self.q_perm[self.q_off[r]:self.q_off[r] +
                                                              self.counts[r]], r, self.group))
                ops.append(dist.P2POp(dist.isend, self.meta_all[self.meta_off[r]:self.meta_off[r] +
                                                                self.meta_len[r]], r, self.group))
        else:
            ops.append(dist.P2POp(dist.irecv, self.q, 0, self.group))
            ops.append(dist.P2POp(dist.irecv, self.meta, 0, self.group))
        if self.world > 1:
            self._exchange(ops)

    def gather(self, out=None):
        """Step part 4: rank 0 returns the outputs [S, Hq, D] in batch order (in ``out``
        when given, else in a buffer of its own that the next step overwrites); others None."""
        import torch
        import torch.distributed as dist

        dst = (self.out_batch if out is None else out) if self.rank == 0 else None
        if self.exchange == "peer":
            from . import _native

            lib = _native.lib()
            if self.rank != 0:
                _native.check(lib.ouro_shard_signal(self._done_flag, self.step_no,
                                                    self._stream()), "shard signal")
                return None
            _native.check(lib.ouro_shard_collect(
                self._own + 64, self.world - 1, 8, self.step_no, self.timeout_ns,
                self.out_perm.data_ptr(), self.inv.data_ptr(), dst.data_ptr(), self.S,
                self.row_bytes, self.exchange_status.data_ptr(), self._stream()), "shard collect")
            return dst
        ops = []
        if self.rank == 0:
            for r in range(1, self.world):
                ops.append(dist.P2POp(dist.irecv, self.out_perm[self.q_off[r]:self.q_off[r] +
                                                                self.counts[r]], r, self.group))
        else:
            ops.append(dist.P2POp(dist.isend, self.out, 0, self.group))
        if self.world > 1:
            self._exchange(ops)
        if self.rank != 0:
            return None
        torch.index_select(self.out_perm, 0, self.inv, out=dst)
        return dst

    def step(self, run: Callable, q_batch=None, out=None):
        """One decode step: scatter, ``run()`` on every rank, gather (rank 0 gets the rows)."""
        self.scatter(q_batch)
        run()
        return self.gather(out)
