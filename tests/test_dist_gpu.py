"""Sharded decode step on 2 GPUs over NCCL: whole sequences per GPU, Supervisor on rank 0.

Each rank owns one KV pool (caches on its GPU); rank 0 holds both pools'
allocators, builds each rank's page-table slice and query shard, scatters
them, every rank runs the tensor-core decode on its shard, and rank 0 gathers
the rows. Rank 0 checks every gathered row against the oracle (max-abs 2e-2,
mean-abs 2e-3, bf16) and that no kernel reported a status bit. Skipped with
fewer than 2 GPUs. NVLS is off (NCCL_NVLS_ENABLE=0): the test runs plain
NCCL point-to-point traffic only.
"""

import os
import random
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]

pytestmark = pytest.mark.gpu

HQ, HKV, D = 32, 8, 128


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _pool(rank):
    """Deterministic pool of rank `rank`: (BlockTable, heads, lens, k, v) on the CPU."""
    from src.block_table import BlockTable

    rng = random.Random(100 + rank)
    lens = [rng.randint(1, 1500) for _ in range(5 + rank)]
    nblocks = sum(-(-n // 64) for n in lens) + 4
    bt = BlockTable(nblocks)
    ids = [bt.allocate_block() for _ in range(nblocks)]
    rng.shuffle(ids)
    for i in ids:
        bt.free_block(i)
    heads = [bt.allocate_chain(-(-n // 64)) for n in lens]
    g = torch.Generator().manual_seed(200 + rank)
    k = (torch.randn(nblocks, HKV, 64, D, generator=g) * 0.5).bfloat16()
    v = (torch.randn(nblocks, HKV, 64, D, generator=g) * 0.5).bfloat16()
    q = (torch.randn(len(lens), HQ, D, generator=g) * 0.5).bfloat16()
    return bt, heads, lens, k, v, q


def _worker(rank, world, port, result_q):
    sys.path.insert(0, str(ROOT / "ouroboros-triton_b200"))
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch.distributed as dist

    from oracle import attention_oracle as ao
    from src.block_table import build_page_table_array
    from src.dist import sharded_step
    from src.kernels import block_attention as ba

    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=300), device_id=device)
    try:
        _, _, _, k_cpu, v_cpu, _ = _pool(rank)
        k, v = k_cpu.to(device), v_cpu.to(device)
        cos, sin = ao.rope_tables(2048, D, 500000.0)
        cos_d, sin_d = torch.from_numpy(cos).to(device), torch.from_numpy(sin).to(device)
        status = torch.zeros(1, dtype=torch.int32, device=device)

        def compute(q, pt, lens):
            return ba.block_attention_decode(pt, q, k, v, lens, cos_d, sin_d, status=status)

        if rank == 0:
            pools = [_pool(r) for r in range(world)]
            pts = [torch.from_numpy(build_page_table_array(bt, heads)) for bt, heads, *_ in pools]
            q_sh = [p[5].to(device) for p in pools]
            ln_sh = [torch.tensor(p[2], dtype=torch.int32) for p in pools]
            outs = sharded_step(compute, world, rank, device, q_shards=q_sh,
                                pt_shards=[t.to(device) for t in pts],
                                len_shards=[t.to(device) for t in ln_sh])
            errs = []
            for r, (o, p, pt) in enumerate(zip(outs, pools, pts)):
                want = ao.decode_attention(pt.numpy(), p[5].float().numpy(), p[3].float().numpy(),
                                           p[4].float().numpy(), p[2], cos, sin)
                e = np.abs(o.float().cpu().numpy() - want)
                errs.append((float(e.max()), float(e.mean())))
            torch.cuda.synchronize(device)
            result_q.put(("done", errs, int(status.item())))
        else:
            sharded_step(compute, world, rank, device)
            torch.cuda.synchronize(device)
            if int(status.item()) != 0:
                result_q.put(("status", rank, int(status.item())))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_sharded_decode_two_gpus_nccl():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    msgs = []
    while not q.empty():
        msgs.append(q.get(timeout=5))
    done = [m for m in msgs if m[0] == "done"]
    assert done and not [m for m in msgs if m[0] == "status"], msgs
    _, errs, st = done[0]
    assert st == 0
    for mx, mean in errs:
        assert mx <= 2e-2 and mean <= 2e-3, errs


def _peer_worker(rank, world, port, result_q):
    sys.path.insert(0, str(ROOT / "ouroboros-triton_b200"))
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch.distributed as dist

    from oracle import attention_oracle as ao
    from src.dist import DecodeShards
    from src.kernels import block_attention as ba
    from src.serving import lpt_placement

    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=300), device_id=device)
    sh = None
    try:
        # one batch of 11 sequences placed on the ranks by LPT; every rank's pool from _pool
        pools = [_pool(r) for r in range(world)]
        lens = [n for p in pools for n in p[2]]
        placement = lpt_placement(lens, [0] * world)
        counts = [placement.count(r) for r in range(world)]
        # rank r's pool holds its placed sequences: rebuild pools with those lengths
        from src.block_table import BlockTable, build_page_table_array
        tables = []
        for r in range(world):
            mine = [lens[i] for i in range(len(lens)) if placement[i] == r]
            nb = sum(-(-n // 64) for n in mine) + 3
            bt = BlockTable(nb)
            heads = [bt.allocate_chain(-(-n // 64)) for n in mine]
            tables.append((nb, mine, build_page_table_array(bt, heads)))
        nb, mine, pt = tables[rank]
        g = torch.Generator().manual_seed(300 + rank)
        k = (torch.randn(nb, HKV, 64, D, generator=g) * 0.5).bfloat16()
        v = (torch.randn(nb, HKV, 64, D, generator=g) * 0.5).bfloat16()
        kd, vd = k.to(device), v.to(device)
        cos, sin = ao.rope_tables(2048, D, 500000.0)
        cos_d, sin_d = torch.from_numpy(cos).to(device), torch.from_numpy(sin).to(device)
        sh = DecodeShards(world, rank, device, q_heads=HQ, head_dim=D, dtype=torch.bfloat16,
                          placement=placement if rank == 0 else None,
                          widths=[t[2].shape[1] for t in tables] if rank == 0 else None,
                          exchange="peer")
        if rank == 0:
            sh.set_meta([t[1] for t in tables], [torch.from_numpy(t[2]) for t in tables])
        status = torch.zeros(1, dtype=torch.int32, device=device)
        call = ba.DecodeCall(sh.page_table, sh.q, kd, vd, sh.seq_lens, cos_d, sin_d,
                             out_ptr=sh.out_ptr, validate=False, status=status)
        gq = torch.Generator().manual_seed(7)
        errs = []
        for step in range(3):  # every step new queries; rows checked on rank 0
            q = (torch.randn(len(lens), HQ, D, generator=gq) * 0.5).bfloat16()
            out = sh.step(call.launch, q.to(device) if rank == 0 else None)
            if rank == 0:
                got = out.float().cpu().numpy()
            if rank == 0:  # rank 0 rebuilds every pool's values (same seeds) for the oracle
                for r in range(world):
                    nbr, mine_r, pt_r = tables[r]
                    gr = torch.Generator().manual_seed(300 + r)
                    kr = (torch.randn(nbr, HKV, 64, D, generator=gr) * 0.5).bfloat16()
                    vr = (torch.randn(nbr, HKV, 64, D, generator=gr) * 0.5).bfloat16()
                    idx = sh.shard_of(r)
                    want = ao.decode_attention(pt_r, q[idx].float().numpy(), kr.float().numpy(),
                                               vr.float().numpy(), mine_r, cos, sin)
                    e = np.abs(got[idx] - want)
                    errs.append((float(e.max()), float(e.mean())))
        torch.cuda.synchronize(device)
        st = [int(status.item()), int(sh.exchange_status.item())]
        if rank == 0:
            result_q.put(("done", errs, st, counts))
        elif any(st):
            result_q.put(("status", rank, st))
    finally:
        if sh is not None:
            sh.close()
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_decode_shards_peer_exchange_two_gpus():
    """DecodeShards with the peer-memory exchange: rank 0 publishes, the worker fetches over
    NVLink and its decode writes into rank 0's buffer; three steps, every row vs the oracle."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    msgs = []
    while not q.empty():
        msgs.append(q.get(timeout=5))
    done = [m for m in msgs if m[0] == "done"]
    assert done and not [m for m in msgs if m[0] == "status"], msgs
    _, errs, st, counts = done[0]
    assert st == [0, 0] and min(counts) >= 1
    assert len(errs) == 6
    for mx, mean in errs:
        assert mx <= 2e-2 and mean <= 2e-3, errs
