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


def _shards_worker(rank, world, port, result_q):
    sys.path.insert(0, str(ROOT / "ouroboros-triton_b200"))
    from src.dist import DecodeShards
    from src.serving import lpt_placement

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        S, hq, d = 11, 2, 4
        g = torch.Generator().manual_seed(3)
        lens = torch.randint(1, 900, (S,), generator=g, dtype=torch.int32)
        widths = [15, 9, 12][:world]
        placement = lpt_placement(lens.tolist(), [0] * world) if rank == 0 else None
        sh = DecodeShards(world, rank, torch.device("cpu"), q_heads=hq, head_dim=d,
                          dtype=torch.float32, placement=placement,
                          widths=widths if rank == 0 else None)
        if rank == 0:
            # rank r's page-table rows: row i of the shard holds (batch index * 100 + column)
            pts = [torch.tensor([[b * 100 + c for c in range(widths[r])] for b in sh.shard_of(r)],
                                dtype=torch.int32) for r in range(world)]
            sh.set_meta([lens[sh.shard_of(r)] for r in range(world)], pts)

        def run():  # stand-in decode: every input shows up in the row
            sh.out.copy_(sh.q * 2 + sh.page_table[:, -1:, None].float()
                         + sh.seq_lens[:, None, None].float())

        results = []
        for step in range(3):  # repeated steps reuse every buffer
            q = (torch.arange(S * hq * d, dtype=torch.float32).view(S, hq, d) + 1000 * step
                 if rank == 0 else None)
            out = sh.step(run, q)
            if rank == 0:
                last_col = torch.tensor([b * 100 + widths[placement[b]] - 1 for b in range(S)],
                                        dtype=torch.float32)
                want = q * 2 + last_col[:, None, None] + lens[:, None, None].float()
                results.append(bool(torch.equal(out, want)))
        if rank == 0:
            result_q.put((all(results), sh.counts))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_decode_shards_routes_every_sequence_and_restores_batch_order(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_shards_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    ok, counts = q.get(timeout=5)
    assert ok and sum(counts) == 11 and min(counts) >= 1, counts
