"""Scatter -> compute -> gather routing of the sharded decode step on 2 gloo CPU ranks.

The compute is a stand-in (a fixed function of the inputs), because decode
itself runs only on the GPU; the test checks that every rank receives exactly
its shard (queries, page-table slice, lengths) and that rank 0 gets the rows
back in rank order with the padding removed. It also checks that a rank that
dies before the step makes the survivor's collective fail with an error
instead of hanging (short process-group timeout).
"""

import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _compute(q, pt, lens):
    # stand-in for decode: depends on every input so misrouting shows up
    return q * 2 + pt[:, :1, None].float() + lens[:, None, None].float()


def _worker(rank, world, port, result_q):
    sys.path.insert(0, str(ROOT / "ouroboros-triton_b200"))
    from src.dist import sharded_step

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    try:
        if rank == 0:
            q = [torch.arange(3 * 2 * 4, dtype=torch.float32).view(3, 2, 4),
                 torch.arange(5 * 2 * 4, dtype=torch.float32).view(5, 2, 4) + 100]
            pt = [torch.tensor([[7, 8, -1], [3, -1, -1], [1, 2, 4]], dtype=torch.int32),
                  torch.arange(5, dtype=torch.int32).view(5, 1)]
            ln = [torch.tensor([130, 64, 190], dtype=torch.int32),
                  torch.tensor([1, 2, 3, 4, 5], dtype=torch.int32)]
            outs = sharded_step(_compute, world, rank, torch.device("cpu"), q_shards=q,
                                pt_shards=pt, len_shards=ln)
            want = [_compute(a, b, c) for a, b, c in zip(q, pt, ln)]
            ok = all(torch.equal(o, w) for o, w in zip(outs, want))
            result_q.put(("ok" if ok else "mismatch", [tuple(o.shape) for o in outs]))
        else:
            sharded_step(_compute, world, rank, torch.device("cpu"))
    finally:
        dist.destroy_process_group()


def test_sharded_step_routes_and_gathers_on_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    status, shapes = q.get(timeout=5)
    assert status == "ok" and shapes == [(3, 2, 4), (5, 2, 4)]


def _dead_rank_worker(rank, world, port, result_q):
    sys.path.insert(0, str(ROOT / "ouroboros-triton_b200"))
    from src.dist import sharded_step

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)   # the rank leaves between steps, with nothing in flight
    try:
        sharded_step(_compute, world, rank, torch.device("cpu"),
                     q_shards=[torch.zeros(1, 1, 2)] * 2,
                     pt_shards=[torch.zeros(1, 1, dtype=torch.int32)] * 2,
                     len_shards=[torch.ones(1, dtype=torch.int32)] * 2)
        result_q.put("no error")
    except Exception as exc:  # noqa: BLE001
        result_q.put(f"error: {type(exc).__name__}")


def test_dead_rank_surfaces_as_an_error_not_a_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dead_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    msg = q.get(timeout=5)
    assert msg.startswith("error"), msg
