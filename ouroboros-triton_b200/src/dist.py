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
