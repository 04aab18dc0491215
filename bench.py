"""Paged-decode benchmark: tokens/s and achieved HBM GB/s on B200.

Workload (one GPU): GQA paged decode, Llama-3-70B attention shape — 256
sequences, 64 query heads, 8 KV heads, head_dim 128, bf16, context lengths
uniform in [8192, 32768], 64-token blocks scattered over a per-GPU pool sized
to the shard + 5 %, Q/K/V ~ 0.5 N(0, 1), RoPE base 500000. A step decodes
one token for every sequence (split-K decode + combine).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

The batch is the Supervisor's: 256 sequences at every N (strong scaling).
Under torchrun (N > 1) the Supervisor (rank 0) places whole sequences on the
ranks by longest-processing-time on token count, and every step sends each
rank its queries and metadata and gathers the output rows back over NCCL
inside the timed region; time = max over ranks. The line also carries the
weak-scaling figure (256 sequences per GPU, N > 1) and the chunked-prefill
measurement (8 x 4096-token prompts in 512-token chunks per GPU) as
sub-objects. `--impl reference` times the CPU path (the numpy restatement of
the reference's dense_reference, one query row per sequence) on this host's
cores, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import random
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "ouroboros-triton_b200"))
sys.path.insert(0, str(ROOT))

WORKLOAD = dict(workload="gqa_paged_decode_llama3_70b", seqs_per_gpu=256, q_heads=64,
                kv_heads=8, head_dim=128, dtype="bf16", ctx_min=8192, ctx_max=32768,
                block_tokens=64, rope_base=500000.0, pool_headroom=0.05)
METRIC = "paged-decode attn tokens/s + achieved HBM GB/s vs peak at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def _lens(seed: int, n: int):
    rng = random.Random(seed)
    return [rng.randint(WORKLOAD["ctx_min"], WORKLOAD["ctx_max"]) for _ in range(n)]


def _dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


class ClockSampler:
    """SM clocks and throttle reasons sampled every 10 ms during the timed region.

    Reads NVML (the library behind nvidia-smi) from a background thread;
    falls back to an `nvidia-smi -lms` subprocess when NVML is unavailable.
    """

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = None
        self._thread = None
        self._smi = None

    def __enter__(self):
        import threading
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByIndex(self.gpu)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            self._stop = threading.Event()

            def loop():
                while not self._stop.is_set():
                    try:
                        self.samples.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
                        bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                        for name, bit in self.REASONS.items():
                            if bits & bit:
                                self.reasons.add(name)
                    except Exception:  # noqa: BLE001 - sampling must never break the bench
                        pass
                    self._stop.wait(0.01)

            self._thread = threading.Thread(target=loop, daemon=True)
            self._thread.start()
        except Exception:  # noqa: BLE001
            self._thread = None
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)

    def summary(self):
        if self._thread is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "samples": 0,
                    "reasons": ["NVML unavailable"]}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "samples": len(self.samples),
                "reasons": sorted(self.reasons)}


# ---------------------------------------------------------------------------
# CPU path (reference arm and cpu_baseline): the oracle's decode restatement
# ---------------------------------------------------------------------------

def _cpu_decode_sample(n_seqs: int, threads: int, seed: int):
    """Times the numpy decode restatement on n_seqs sequences of the workload shape.

    Returns (seconds, tokens decoded). Each sequence gets its own scattered
    paged caches (same shapes and value distribution as the GPU workload).
    """
    import numpy as np
    from concurrent.futures import ThreadPoolExecutor

    from oracle import attention_oracle as ao

    W = WORKLOAD
    lens = _lens(seed, n_seqs)
    hkv, hq, d = W["kv_heads"], W["q_heads"], W["head_dim"]
    max_b = -(-W["ctx_max"] // 64)
    cos, sin = ao.rope_tables(max_b * 64, d, W["rope_base"])
    rng = np.random.default_rng(seed)
    jobs = []
    for n in lens:
        nb = -(-n // 64)
        perm = rng.permutation(nb + 8)[:nb]
        k = (rng.standard_normal((nb + 8, hkv, 64, d), dtype=np.float32) * 0.5).astype(np.float16)
        v = (rng.standard_normal((nb + 8, hkv, 64, d), dtype=np.float32) * 0.5).astype(np.float16)
        pt = np.full((1, max_b), -1, np.int32)
        pt[0, :nb] = perm
        q = (rng.standard_normal((1, hq, d), dtype=np.float32) * 0.5).astype(np.float16)
        jobs.append((pt, q, k, v, [n]))

    def one(job):
        pt, q, k, v, ln = job
        return ao.decode_attention(pt, q, k, v, ln, cos, sin)

    t0 = time.perf_counter()
    with ThreadPoolExecutor(max_workers=threads) as ex:
        list(ex.map(one, jobs))
    return time.perf_counter() - t0, n_seqs


def run_reference(args):
    world, rank, _ = _dist_env()
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    per_step = max(1, min(threads, 16))
    for i in range(args.warmup):
        _cpu_decode_sample(per_step, threads, 1000 + i)
    secs, toks = 0.0, 0
    for i in range(args.steps):
        s, t = _cpu_decode_sample(per_step, threads, 2000 + i)
        secs += s
        toks += t
    value = toks / secs
    sample = (f"{per_step} sequences per step of the {WORKLOAD['workload']} shape "
              f"(lens U[{WORKLOAD['ctx_min']},{WORKLOAD['ctx_max']}]), numpy fp32 row-restricted "
              "restatement of the reference's dense_reference (its full TxT form is infeasible "
              "at these lengths)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * secs / max(args.steps, 1), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": dict({k: x for k, x in WORKLOAD.items() if k != "seqs_per_gpu"},
                       seqs=WORKLOAD["seqs_per_gpu"],
                       parallelism="host cores of rank 0 (the reference path has no GPU "
                                   "sharding)", l2_flush="inputs>L2"),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# GPU path
# ---------------------------------------------------------------------------

def _build_shard(torch, device, seed: int, n_seqs: int, len_seed: int | None = None):
    import numpy as np

    from oracle import attention_oracle as ao  # RoPE table construction only
    from src.block_table import BlockTable

    W = WORKLOAD
    S, hq, hkv, d = n_seqs, W["q_heads"], W["kv_heads"], W["head_dim"]
    lens = _lens(seed if len_seed is None else len_seed, S)
    need = sum(-(-n // 64) for n in lens)
    pool = int(math.ceil(need * (1 + W["pool_headroom"])))
    bt = BlockTable(pool)
    ids = [bt.allocate_block() for _ in range(pool)]
    random.Random(seed).shuffle(ids)
    for i in ids:
        bt.free_block(i)
    heads = [bt.allocate_chain(-(-n // 64)) for n in lens]
    max_b = -(-W["ctx_max"] // 64)
    pt_host = bt.export_page_table(heads, max_b)
    g = torch.Generator(device=device).manual_seed(seed)
    k = torch.empty((pool, hkv, 64, d), dtype=torch.bfloat16, device=device)
    v = torch.empty_like(k)
    chunk = 4096
    for lo in range(0, pool, chunk):
        hi = min(pool, lo + chunk)
        k[lo:hi] = (torch.randn((hi - lo, hkv, 64, d), generator=g, device=device) * 0.5)
        v[lo:hi] = (torch.randn((hi - lo, hkv, 64, d), generator=g, device=device) * 0.5)
    q = (torch.randn((S, hq, d), generator=g, device=device) * 0.5).to(torch.bfloat16)
    cos, sin = ao.rope_tables(max_b * 64, d, W["rope_base"])
    return dict(lens=lens, pool=pool, table=bt, heads=heads, pt_host=pt_host,
                pt=torch.from_numpy(pt_host).to(device),
                seq_lens=torch.tensor(lens, dtype=torch.int32, device=device),
                k=k, v=v, q=q, cos=torch.from_numpy(cos).to(device),
                sin=torch.from_numpy(sin).to(device))


def _cpu_baseline_leg():
    threads = os.cpu_count() or 1
    n = max(1, min(threads, 16))
    secs, toks = _cpu_decode_sample(n, threads, 77)
    return {"value": toks / secs, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{n} sequences of the workload shape, numpy fp32 row-restricted "
                      "restatement of dense_reference, one thread per sequence"}


def _init_dist(world: int, local: int, timeout_s: int = 120):
    import datetime

    import torch
    import torch.distributed as dist

    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=timeout_s),
                                device_id=torch.device("cuda", local))
    device = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(device)
    return device


def _supervisor_batch(n_seqs: int, world: int):
    """The batch the Supervisor decodes: context lengths (seeded) and their
    longest-processing-time placement over the ranks by token count."""
    from src.serving import lpt_placement

    lens = _lens(1234, n_seqs)
    placement = lpt_placement(lens, [0] * world)
    shards = [[i for i in range(n_seqs) if placement[i] == r] for r in range(world)]
    return lens, placement, shards


def _pool_blocks(lens) -> int:
    need = sum(-(-n // 64) for n in lens)
    return int(math.ceil(need * (1 + WORKLOAD["pool_headroom"])))


def _shard_table(lens, seed: int):
    """One rank's allocator, built by the Supervisor: every block allocated, freed in a
    seeded shuffled order (scattered chains), then one chain per sequence."""
    from src.block_table import BlockTable

    pool = _pool_blocks(lens)
    bt = BlockTable(pool)
    ids = [bt.allocate_block() for _ in range(pool)]
    random.Random(seed).shuffle(ids)
    for i in ids:
        bt.free_block(i)
    heads = [bt.allocate_chain(-(-n // 64)) for n in lens]
    width = max(-(-n // 64) for n in lens)
    return bt, heads, bt.export_page_table(heads, width), width


def _random_pool(torch, device, pool: int, seed: int):
    W = WORKLOAD
    g = torch.Generator(device=device).manual_seed(seed)
    k = torch.empty((pool, W["kv_heads"], 64, W["head_dim"]), dtype=torch.bfloat16, device=device)
    v = torch.empty_like(k)
    for lo in range(0, pool, 4096):
        hi = min(pool, lo + 4096)
        k[lo:hi] = torch.randn((hi - lo,) + tuple(k.shape[1:]), generator=g, device=device) * 0.5
        v[lo:hi] = torch.randn((hi - lo,) + tuple(k.shape[1:]), generator=g, device=device) * 0.5
    return k, v


def run_ours(args):
    """The headline line: GQA paged decode of one 256-sequence batch owned by the Supervisor.

    The Supervisor (rank 0) places the batch's whole sequences on the N ranks by
    longest-processing-time on token count and owns every rank's allocator; rank r
    holds its pool's K/V. A step is the Supervisor's decode of the batch: permute the
    queries into shard order, send each rank its queries and metadata (lengths and
    page-table rows), decode every shard, gather the rows back and restore the batch
    order (src.dist.DecodeShards), all inside the timed region. N = 1 runs the same
    step with no collective. Strong scaling: the batch is 256 sequences at every N.
    """
    import torch
    import torch.distributed as dist

    from oracle import attention_oracle as ao  # RoPE table construction only
    from src.dist import DecodeShards
    from src.kernels.block_attention import DecodeCall, validate_page_table

    world, rank, local = _dist_env()
    device = _init_dist(world, local)
    # The chunked-prefill leg runs first, before the decode pool (21 GB per GPU at N = 1)
    # is allocated: measured after the decode legs, with their buffers still held, the
    # same prefill ran ~12 % slower on some boxes (and at full speed once they were freed).
    pre = _prefill_leg(args, world, rank, device) if not args.no_prefill else None
    W = WORKLOAD
    S, hq, hkv, d = (args.seqs if args.seqs > 0 else W["seqs_per_gpu"]), W["q_heads"], \
        W["kv_heads"], W["head_dim"]
    lens, placement, shards = _supervisor_batch(S, world)
    my_lens = [lens[i] for i in shards[rank]]
    tables = None
    if rank == 0:  # the Supervisor's allocators, one per rank's pool
        tables = [_shard_table([lens[i] for i in shards[r]], 1234 + r) for r in range(world)]
    sh = DecodeShards(world, rank, device, q_heads=hq, head_dim=d, dtype=torch.bfloat16,
                      placement=placement if rank == 0 else None,
                      widths=[t[3] for t in tables] if rank == 0 else None,
                      exchange=args.exchange)
    if sh.n != len(my_lens):
        raise RuntimeError(f"rank {rank}: shard size {sh.n} != placement {len(my_lens)}")
    if rank == 0:
        sh.set_meta([[lens[i] for i in shards[r]] for r in range(world)],
                    [torch.from_numpy(t[2]) for t in tables])
    pool = _pool_blocks(my_lens)
    k, v = _random_pool(torch, device, pool, 1234 + rank)
    max_b = -(-W["ctx_max"] // 64)
    cos_np, sin_np = ao.rope_tables(max_b * 64, d, W["rope_base"])
    cos, sin = torch.from_numpy(cos_np).to(device), torch.from_numpy(sin_np).to(device)
    q_batch = None
    if rank == 0:
        g = torch.Generator(device=device).manual_seed(99)
        q_batch = (torch.randn((S, hq, d), generator=g, device=device) * 0.5).to(torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    my_blocks = sum(-(-n // 64) for n in my_lens)
    call = DecodeCall(sh.page_table, sh.q, k, v, sh.seq_lens, cos, sin, out_ptr=sh.out_ptr,
                      validate=False, split_blocks=args.split_blocks, kernel=args.kernel,
                      status=status, total_blocks=my_blocks, max_seq_blocks=sh.width)
    plan = call.plan
    stream = torch.cuda.current_stream(device)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)

    sh.step(call.launch, q_batch)  # first step: the metadata has arrived, check it
    validate_page_table(sh.page_table, sh.seq_lens, pool)
    for _ in range(max(args.warmup, 3)):
        sh.step(call.launch, q_batch)
    barrier()
    n_ev = args.steps
    k0 = [torch.cuda.Event(enable_timing=True) for _ in range(n_ev)]
    k1 = [torch.cuda.Event(enable_timing=True) for _ in range(n_ev)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def launch_timed(i):
        def run():
            k0[i].record(stream)
            call.launch()
            k1[i].record(stream)
        return run

    # The step time comes from steps with nothing but the work on the stream; the decode
    # kernels' own time from the same K steps again with events around the decode launches
    # (an event between two kernels keeps the second from starting early, as the
    # programmatic launch chain of the exchange and decode kernels otherwise lets it).
    with ClockSampler(device.index) as clk:
        barrier()
        start.record(stream)
        for i in range(args.steps):
            sh.step(call.launch, q_batch)
        stop.record(stream)
        barrier()
    # The instrumented pass starts from the same power state as the timed one: after ~60 ms
    # of back-to-back decode the power limiter (sw_power_cap) can engage, and without a
    # pause the second pass measured 1-3 % slower kernels than the first.
    time.sleep(1.0)
    barrier()
    start2, stop2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start2.record(stream)
    for i in range(args.steps):
        sh.step(launch_timed(i), q_batch)
    stop2.record(stream)
    barrier()
    ms = start.elapsed_time(stop)
    kern_ms = sum(a.elapsed_time(b) for a, b in zip(k0, k1)) / args.steps
    ev_step_ms = start2.elapsed_time(stop2) / args.steps
    t = torch.tensor([ms, kern_ms, ev_step_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max, kern_max, ev_step_max = float(t[0]), float(t[1]), float(t[2])
    step_ms = ms_max / args.steps
    value = S * args.steps / (ms_max / 1000.0)
    kv_bytes_all = sum(lens) * hkv * d * 2 * 2
    kv_bytes_mine = sum(my_lens) * hkv * d * 2 * 2
    # this rank's decode kernels (decode + combine) per launch, timed inside the region
    achieved_mine = kv_bytes_mine / (kern_ms / 1000.0) / 1e9

    # every rank's kernel status and decode rate, to the Supervisor
    st_all = [torch.zeros(2, dtype=torch.float64, device=device) for _ in range(world)]
    mine_t = torch.tensor([float(status.item()), achieved_mine], dtype=torch.float64,
                          device=device)
    if world > 1:
        dist.all_gather(st_all, mine_t)
    else:
        st_all = [mine_t]
    statuses = [int(x[0]) for x in st_all]
    rates = [float(x[1]) for x in st_all]
    xst = torch.tensor([float(sh.exchange_status.item())], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(xst, op=dist.ReduceOp.MAX)
    check = _check_gathered_rows(torch, dist, sh, world, rank, lens, shards, tables, k, v,
                                 cos_np, sin_np, q_batch)
    if rank == 0:
        check["kernel_status"] = statuses
        check["exchange_status"] = int(xst.item())
    if any(statuses):
        print(f"rank {rank}: decode kernels reported status {statuses}", file=sys.stderr)

    e2e = _e2e_sharded(torch, dist, sh, call, world, rank, device, q_batch, args)
    weak = _weak_scaling_leg(torch, dist, world, rank, device, args) if world > 1 else None
    serv = None
    if not args.no_serving:
        if args.serving_rate <= 0:
            args.serving_rate = 4096.0
        serv = _serving_leg(args, world, rank, device)
    sapi = (_supervisor_api_leg(args, device)
            if (world == 1 and not args.no_supervisor_api) else None)
    refk = (_reference_kernel_leg(args, device)
            if (rank == 0 and world == 1 and not args.no_reference_kernel) else None)
    cpu = _cpu_baseline_leg() if (rank == 0 and world == 1 and not args.no_cpu) else None
    peak, peak_kind = _peaks()
    launches = args.steps * plan["launches"]
    if rank == 0:
        avg_rate = kv_bytes_all / world / (kern_max / 1000.0) / 1e9
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded; random-init K/V/Q, no dataset)",
            "config": dict({k: x for k, x in WORKLOAD.items() if k != "seqs_per_gpu"}, seqs=S,
                           parallelism=(f"dp{world}: the Supervisor (rank 0) places whole "
                                        "sequences by LPT on tokens; queries, lengths and "
                                        "page-table rows go out and outputs come back inside "
                                        "every step" if world > 1 else
                                        "dp1 (the Supervisor's batch on one GPU)"),
                           exchange=(("peer memory over NVLink (CUDA IPC; fetch / signal / "
                                      "collect kernels, bounded flag waits)"
                                      if sh.exchange == "peer" else "NCCL point-to-point")
                                     if world > 1 else None),
                           shard_sizes=sh.counts,
                           shard_tokens=[sum(lens[i] for i in shards[r]) for r in range(world)],
                           l2_flush="inputs>L2 (K+V %.1f GB per GPU)" % (kv_bytes_all / world / 1e9),
                           split_blocks=None if plan["stream_k"] else plan["split_blocks"],
                           max_splits=None if plan["stream_k"] else plan["max_splits"],
                           stream_k_ctas=plan["max_splits"] if plan["stream_k"] else None,
                           kernel=("tensor_cores_stream_k" if plan["stream_k"] else
                                   "tensor_cores" if plan["tensor_cores"] else "cuda_cores")),
            "roofline": {"bound": "hbm", "achieved": avg_rate, "peak": peak, "unit": "GB/s",
                         "frac": avg_rate / peak, "traffic": _traffic_from_profile(world),
                         "peak_source": peak_kind,
                         "algorithmic_bytes_per_launch": kv_bytes_all // world,
                         "per_rank_GB/s": rates,
                         "note": "prep + decode + merge launches timed with CUDA events "
                                 "around them in K more steps, 1 s after the timed ones; "
                                 "K+V bytes once per KV head; "
                                 "achieved = the batch's bytes / N over the slowest rank's "
                                 "kernel time"},
            "step_breakdown_ms": {"step": step_ms,
                                  "step_with_kernel_events": ev_step_max,
                                  "decode_kernels_max_rank": kern_max,
                                  "outside_kernels": ev_step_max - kern_max},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clk.summary(),
            "check": check,
        }
        if weak is not None:
            line["weak_scaling"] = weak
        if pre is not None:
            line["prefill"] = pre
        if serv is not None:
            line["serving"] = serv
        if sapi is not None:
            line["supervisor_api"] = sapi
        if refk is not None:
            line["reference_kernel"] = refk
        print(json.dumps(line), flush=True)
    sh.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def _check_gathered_rows(torch, dist, sh, world, rank, lens, shards, tables, k, v, cos_np,
                         sin_np, q_batch):
    """The Supervisor checks rows it gathered from EVERY rank against the oracle.

    Per rank the two shortest sequences are checked: the rank sends the K/V blocks of
    their chains (in chain order) to rank 0, which recomputes those rows with the numpy
    oracle and compares them with the rows of the last gathered step.
    """
    import numpy as np

    from oracle import attention_oracle as ao

    picks = [sorted(range(len(shards[r])), key=lambda j: (lens[shards[r][j]], j))[:2]
             for r in range(world)]
    blocks = [[-(-lens[shards[r][j]] // 64) for j in picks[r]] for r in range(world)]
    mine = picks[rank]
    pt = sh.page_table[mine].cpu().numpy()
    ids = [int(pt[i, b]) for i in range(len(mine)) for b in range(blocks[rank][i])]
    sel = torch.tensor(ids, dtype=torch.int64, device=k.device)
    kb, vb = k.index_select(0, sel).contiguous(), v.index_select(0, sel).contiguous()
    res = None
    if rank == 0:
        errs = []
        got_all = sh.out_batch.float().cpu().numpy()  # the last timed step's gathered rows
        for r in range(world):
            nb = sum(blocks[r])
            if r == 0:
                kr, vr = kb, vb
            else:
                kr = torch.empty((nb,) + tuple(k.shape[1:]), dtype=k.dtype, device=k.device)
                vr = torch.empty_like(kr)
                dist.recv(kr, src=r)
                dist.recv(vr, src=r)
            kn, vn = kr.float().cpu().numpy(), vr.float().cpu().numpy()
            off = 0
            for j, nbj in zip(picks[r], blocks[r]):
                b = shards[r][j]
                ptj = np.full((1, nbj), -1, np.int32)
                ptj[0, :] = np.arange(off, off + nbj, dtype=np.int32)
                q = q_batch[b:b + 1].float().cpu().numpy()
                want = ao.decode_attention(ptj, q, kn, vn, [lens[b]], cos_np, sin_np)
                e = np.abs(got_all[b:b + 1] - want)
                errs.append((r, b, float(e.max()), float(e.mean())))
                off += nbj
        mx = max(e[2] for e in errs)
        mean = float(np.mean([e[3] for e in errs]))
        res = {"rows": len(errs), "per_rank_rows": [list(p) for p in picks],
               "max_abs": mx, "mean_abs": mean,
               "per_rank_max_abs": [max(e[2] for e in errs if e[0] == r) for r in range(world)],
               "tolerance": {"max_abs": 2e-2, "mean_abs": 2e-3},
               "ok": bool(mx <= 2e-2 and mean <= 2e-3)}
    else:
        dist.send(kb, dst=0)
        dist.send(vb, dst=0)
    torch.cuda.synchronize(k.device)
    return res


def _e2e_sharded(torch, dist, sh, call, world, rank, device, q_batch, args):
    """The same step through the public API from host buffers: every step rank 0 uploads the
    batch's queries and the Supervisor's metadata (every shard's lengths and page-table rows)
    from pinned memory and reads the batch's output rows back. Two buffer sets and one
    stream per copy direction, so uploads and read-backs overlap neighbouring steps."""
    stream = torch.cuda.current_stream(device)
    steps = max(5, min(args.steps, 20))
    h2d = d2h = 0
    if rank == 0:
        q_host = q_batch.cpu().pin_memory()
        meta_host = sh.meta_all.cpu().pin_memory()
        out_host = [torch.empty_like(q_host).pin_memory() for _ in range(2)]
        ins = [(torch.empty_like(q_batch), torch.empty_like(sh.meta_all)) for _ in range(2)]
        outs = [torch.empty_like(q_batch) for _ in range(2)]
        h2d = q_host.numel() * q_host.element_size() + meta_host.numel() * 4
        d2h = out_host[0].numel() * out_host[0].element_size()
        up, back = torch.cuda.Stream(device), torch.cuda.Stream(device)
        h2d_done = [torch.cuda.Event() for _ in range(2)]
        used_done = [torch.cuda.Event() for _ in range(2)]
        d2h_done = [torch.cuda.Event() for _ in range(2)]
        used = [False, False]

    def step(i):
        if rank != 0:
            sh.step(call.launch)
            return
        b = i & 1
        qd, md = ins[b]
        with torch.cuda.stream(up):
            if used[b]:
                up.wait_event(used_done[b])  # step i - 2 has consumed buffer set b
            qd.copy_(q_host, non_blocking=True)
            md.copy_(meta_host, non_blocking=True)
            h2d_done[b].record(up)
        stream.wait_event(h2d_done[b])
        if used[b]:
            stream.wait_event(d2h_done[b])  # step i - 2's rows have left outs[b]
        sh.meta_all.copy_(md, non_blocking=True)
        sh.step(call.launch, qd, out=outs[b])
        used_done[b].record(stream)
        with torch.cuda.stream(back):
            back.wait_event(used_done[b])
            out_host[b].copy_(outs[b], non_blocking=True)
            d2h_done[b].record(back)
        used[b] = True

    for i in range(3):
        step(i)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    if rank == 0:
        up.wait_event(e0)  # the first upload starts inside the timed region
    for i in range(steps):
        step(i)
    if rank == 0:
        stream.wait_stream(back)  # the last read-back is inside the timed region
    e1.record(stream)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    te = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    return {"value": sum(sh.counts) * steps / (float(te.item()) / 1000.0), "unit": "tokens/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": steps}


def _weak_scaling_leg(torch, dist, world, rank, device, args):
    """Secondary figure under torchrun: every rank decodes its own 256-sequence batch
    (same lengths on every rank, its own placement and values), no collective in the
    timed loop; value = all ranks' sequences per step / the slowest rank's time."""
    from src.kernels.block_attention import DecodeCall

    W = WORKLOAD
    shd = _build_shard(torch, device, seed=1234 + rank, n_seqs=W["seqs_per_gpu"], len_seed=1234)
    call = DecodeCall(shd["pt"], shd["q"], shd["k"], shd["v"], shd["seq_lens"], shd["cos"],
                      shd["sin"], validate=True, split_blocks=args.split_blocks,
                      kernel=args.kernel, total_blocks=sum(-(-n // 64) for n in shd["lens"]),
                      max_seq_blocks=shd["pt"].shape[1])
    for _ in range(3):
        call.launch()
    torch.cuda.synchronize(device)
    dist.barrier()
    s = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(args.steps):
        call.launch()
    e1.record(s)
    torch.cuda.synchronize(device)
    t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    del shd, call
    torch.cuda.empty_cache()
    return {"seqs_per_gpu": W["seqs_per_gpu"], "scaling": "weak",
            "value": world * W["seqs_per_gpu"] * args.steps / (ms / 1000.0), "unit": "tokens/s",
            "ms_per_step": ms / args.steps,
            "note": "every rank its own 256-sequence batch; no collective in the timed loop"}


def _spot_check(torch, sh, out):
    """Max-abs error of 4 sequences' rows vs the fp32 oracle (kept cheap)."""
    import numpy as np

    from oracle import attention_oracle as ao

    idx = [0, 1, 2, 3]
    pt = sh["pt_host"][idx]
    used = sorted({int(x) for x in pt.reshape(-1) if x >= 0})
    remap = {p: i for i, p in enumerate(used)}
    pt_small = np.vectorize(lambda x: remap.get(int(x), -1))(pt).astype(np.int32)
    sel = torch.tensor(used, device=sh["k"].device)
    k = sh["k"].index_select(0, sel).float().cpu().numpy()
    v = sh["v"].index_select(0, sel).float().cpu().numpy()
    q = sh["q"][idx].float().cpu().numpy()
    want = ao.decode_attention(pt_small, q, k, v, [sh["lens"][i] for i in idx],
                               sh["cos"].cpu().numpy(), sh["sin"].cpu().numpy())
    got = out[idx].float().cpu().numpy()
    err = np.abs(got - want)
    return {"rows": len(idx), "max_abs": float(err.max()), "mean_abs": float(err.mean())}


def _traffic_from_profile(world: int = 1):
    """DRAM bytes per decode launch on one rank, from the ncu capture of this workload
    (recorded for the 256-sequence batch on one GPU; a rank's launch reads 1/N of it, as
    its K+V bytes are 1/N of the batch's)."""
    p = ROOT / "profiles" / "decode_config3_traffic.json"
    if p.exists():
        try:
            b = json.loads(p.read_text()).get("dram_bytes_per_launch")
            return None if b is None else int(b / world)
        except (ValueError, OSError):
            return None
    return None


PREFILL = dict(workload="chunked_prefill_llama3_8b_attention", prompts=8, prompt_len=4096,
               chunk=512, q_heads=32, kv_heads=8, head_dim=128, dtype="bf16", rope_base=500000.0,
               causal=True)


def _supervisor_api_leg(args, device):
    """The Supervisor's single-process API (``Supervisor.decode_step``) on the headline batch.

    One KVPool on this GPU; ``admit_many`` places the 256 sequences (LPT, one pool), the
    pool's caches hold seeded synthetic K/V and each sequence's length is set as if its
    tokens had been appended (20 GB through the append kernel would need as much staging).
    Each step is one ``decode_step(rids, q)`` call: device page tables kept between calls,
    lengths uploaded, the shard launched through the pool's stateless worker and the rows
    returned in request order. CUDA events around the calls (host work included); two rows
    checked against the oracle.
    """
    import numpy as np
    import torch

    from oracle import attention_oracle as ao
    from src.serving import KVPool, Supervisor

    W = WORKLOAD
    S = args.seqs if args.seqs > 0 else W["seqs_per_gpu"]
    lens = _lens(1234, S)
    max_b = -(-W["ctx_max"] // 64)
    pool = KVPool(device=device, num_blocks=_pool_blocks(lens), kv_heads=W["kv_heads"],
                  head_dim=W["head_dim"], dtype=torch.bfloat16, max_positions=max_b * 64,
                  rope_base=W["rope_base"])
    g = torch.Generator(device=device).manual_seed(321)
    pool.k_cache.normal_(0.0, 0.5, generator=g)
    pool.v_cache.normal_(0.0, 0.5, generator=g)
    sup = Supervisor(pools=[pool])
    rids = sup.admit_many(lens)
    for r, n in zip(rids, lens):
        sup.seqs[r].length = n
    q = (torch.randn((S, W["q_heads"], W["head_dim"]), generator=g, device=device) * 0.5
         ).to(torch.bfloat16)
    for _ in range(max(args.warmup, 3)):
        out = sup.decode_step(rids, q)
    torch.cuda.synchronize(device)
    stream = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        out = sup.decode_step(rids, q)
    e1.record(stream)
    torch.cuda.synchronize(device)
    ms = e0.elapsed_time(e1) / args.steps
    errs = []
    cos_np, sin_np = pool.cos.cpu().numpy(), pool.sin.cpu().numpy()
    for i in sorted(range(S), key=lambda j: (lens[j], j))[:2]:
        st = sup.seqs[rids[i]]
        nb = -(-lens[i] // 64)
        ids = torch.tensor(pool.table.page_table_row(st.head)[:nb], dtype=torch.int64,
                           device=device)
        kn = pool.k_cache.index_select(0, ids).float().cpu().numpy()
        vn = pool.v_cache.index_select(0, ids).float().cpu().numpy()
        want = ao.decode_attention(np.arange(nb, dtype=np.int32)[None], q[i:i + 1].float().cpu()
                                   .numpy(), kn, vn, [lens[i]], cos_np, sin_np)
        errs.append(np.abs(out[i:i + 1].float().cpu().numpy() - want))
    err = np.concatenate([e.ravel() for e in errs])
    del sup, pool, q, out
    torch.cuda.empty_cache()
    return {
        "metric": "paged-decode attn tokens/s through Supervisor.decode_step (one process, "
                  "one pool)",
        "value": S / (ms / 1000.0), "unit": "tokens/s", "ms_per_step": ms,
        "steps": args.steps,
        "check": {"rows": 2, "max_abs": float(err.max()), "mean_abs": float(err.mean()),
                  "tolerance": {"max_abs": 2e-2, "mean_abs": 2e-3},
                  "ok": bool(err.max() <= 2e-2 and err.mean() <= 2e-3)},
    }


def _prefill_measure(args, world: int, rank: int, device):
    """Chunked prefill: every 512-token chunk of 8 x 4096-token prompts, causal, GQA 32/8.

    A step is one full pass (8 chunk launches, each over all 8 prompts) with the prompts' K/V
    already resident in the paged cache; FLOPs = 4 * D * Hq * sum_p sum_i (i + 1). Under
    torchrun every rank prefills its own 8 prompts on its GPU (whole prompts shard, no
    collective in the data path): weak scaling, time = max over ranks. Returns the line.
    """
    import torch
    import torch.distributed as dist

    from oracle import attention_oracle as ao  # RoPE table construction only
    from src.block_table import BlockTable
    from src.kernels.block_attention import PrefillCall

    P = PREFILL
    S, T, C = P["prompts"], P["prompt_len"], P["chunk"]
    hq, hkv, d = P["q_heads"], P["kv_heads"], P["head_dim"]
    nbp = T // 64
    pool = S * nbp + 16
    bt = BlockTable(pool)
    ids = [bt.allocate_block() for _ in range(pool)]
    random.Random(4).shuffle(ids)
    for i in ids:
        bt.free_block(i)
    heads = [bt.allocate_chain(nbp) for _ in range(S)]
    pt = torch.from_numpy(bt.export_page_table(heads, nbp)).to(device)
    g = torch.Generator(device=device).manual_seed(4 + rank)
    k = (torch.randn(pool, hkv, 64, d, generator=g, device=device) * 0.5).bfloat16()
    v = (torch.randn(pool, hkv, 64, d, generator=g, device=device) * 0.5).bfloat16()
    q = (torch.randn(S, hq, T, d, generator=g, device=device) * 0.5).bfloat16()
    cos, sin = ao.rope_tables(T, d, P["rope_base"])
    cos, sin = torch.from_numpy(cos).to(device), torch.from_numpy(sin).to(device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    calls = []
    workspace = None  # rotated keys: one scratch for the whole prefill, each key rotated once
    for c in range(T // C):
        qc = q[:, :, c * C:(c + 1) * C].contiguous()
        starts = torch.full((S,), c * C, dtype=torch.int32, device=device)
        lens = torch.full((S,), (c + 1) * C, dtype=torch.int32, device=device)
        pt_c = pt.clone()  # the chains as they stand after chunk c was appended
        pt_c[:, (c + 1) * C // 64:] = -1
        calls.append(PrefillCall(pt_c, qc, k, v, starts, lens, cos, sin, causal=True,
                                 kernel=args.kernel if args.kernel != "auto" else "auto",
                                 status=status, workspace=workspace,
                                 krot_valid=torch.full((S,), c * C, dtype=torch.int32),
                                 launch_seq=c))
        workspace = calls[-1].workspace
    flops = 4.0 * d * hq * S * (T * (T + 1) / 2.0)
    steps = args.prefill_steps if args.prefill_steps > 0 else args.steps
    for _ in range(max(args.warmup, 3)):
        for cl in calls:
            cl.launch()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index) as clk:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(steps):
            for cl in calls:
                cl.launch()
        e1.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    ms = e0.elapsed_time(e1) / steps
    if world > 1:  # the job's step time is the slowest rank's
        t = torch.tensor([ms], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    tflops = flops * world / (ms / 1000.0) / 1e12
    peak = None
    pk = ROOT / "MEASURED_PEAKS.json"
    if pk.exists():
        peak = float(json.loads(pk.read_text())["bf16_tflops"])
    # spot check: one head of two prompts' last chunk vs the oracle
    want = ao.prefill_attention(pt[:2].cpu().numpy(), q[:2, :1, T - C:].float().cpu().numpy(),
                                k[:, :1].float().cpu().numpy(), v[:, :1].float().cpu().numpy(),
                                [T - C] * 2, [T] * 2, cos.cpu().numpy(), sin.cpu().numpy())
    got = calls[-1].out[:2, :1].float().cpu().numpy()
    err = abs(got - want)
    per_gpu = tflops / world
    kernel_status = int(status.item())
    del calls, workspace, k, v, q
    torch.cuda.empty_cache()
    return {
        "metric": "chunked-prefill attn TFLOP/s (causal, bf16)", "value": tflops,
        "unit": "TFLOP/s", "n_gpus": world, "steps": steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "dtype": "bf16",
        "data": "synthetic",
        "config": dict(P, prompts_per_gpu=S, chunk_launches=T // C,
                       parallelism=f"dp{world} (whole prompts per GPU)",
                       rotated_keys="one workspace per prefill; each key rotated once (krot_valid)"),
        "tokens_per_s": world * S * T / (ms / 1000.0),
        "roofline": {"bound": "tensor", "achieved": per_gpu, "peak": peak, "unit": "TFLOP/s",
                     "frac": (per_gpu / peak) if peak else None,
                     "peak_source": "measured (bf16_tflops, burst)" if peak else None,
                     "algorithmic_flops_per_step_per_gpu": flops},
        "gpu_launches": steps * (T // C),
        "check": {"max_abs": float(err.max()), "mean_abs": float(err.mean()),
                  "tolerance": {"max_abs": 2e-2, "mean_abs": 2e-3},
                  "ok": bool(err.max() <= 2e-2 and err.mean() <= 2e-3),
                  "kernel_status": kernel_status},
        "clocks": clk.summary(),
    }


def _prefill_leg(args, world: int, rank: int, device):
    """The chunked-prefill measurement as a sub-object of the headline line."""
    line = _prefill_measure(args, world, rank, device)
    return {k: line[k] for k in ("metric", "value", "unit", "ms_per_step", "steps", "scaling",
                                 "tokens_per_s", "roofline", "gpu_launches", "check", "clocks",
                                 "config")}


def run_prefill(args):
    import torch.distributed as dist

    world, rank, local = _dist_env()
    device = _init_dist(world, local)
    line = _prefill_measure(args, world, rank, device)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


REF_KERNEL_SHAPES = {
    "cpu_decode_batch_fp32": dict(seqs=4, lens=[64, 130, 200, 511], heads=8, head_dim=64,
                                  dtype="fp32", pool_blocks=64, rope_base=10000.0, std=1.0),
    "mha_fp16": dict(seqs=32, ctx_min=512, ctx_max=4096, heads=32, head_dim=128, dtype="fp16",
                     pool_blocks=4096, rope_base=10000.0, std=0.5),
}


def _reference_kernel_leg(args, device):
    """The reference's own Triton kernel beside this repository's drop-in block_attention.

    Both through their public entry points on identical inputs: full self-attention
    (every row of every sequence: the reference's entry computes all rows), paged
    q/k/v, RoPE, no bias. Shapes: the CPU-runnable decode batch (fp32; here the
    CUDA-core kernel) and the fp16 MHA shape (32 sequences, lens U[512, 4096], 32
    heads, head_dim 128; here the tcgen05 kernel). Time per call with CUDA events,
    host-side checks included on both sides; FLOPs = 4 H D sum_s T_s^2.
    """
    import torch

    sys.path.insert(0, str(ROOT / "tests"))
    try:
        import reference_kernel

        ref = reference_kernel.load()
    except Exception as exc:  # noqa: BLE001 - the install may be absent
        return {"unavailable": f"{type(exc).__name__}: {exc}"}
    from src.block_table import BlockTable
    from src.kernels.block_attention import block_attention

    out = {"note": "reference = the reference's Triton kernel via its block_attention; ours = "
                   "src.kernels.block_attention.block_attention; full self-attention, every "
                   "row; time per call, host checks included"}
    for name, c in REF_KERNEL_SHAPES.items():
        rng = random.Random(2)
        lens = c.get("lens") or [rng.randint(c["ctx_min"], c["ctx_max"]) for _ in range(c["seqs"])]
        pool, H, D = c["pool_blocks"], c["heads"], c["head_dim"]
        dt = torch.float32 if c["dtype"] == "fp32" else torch.float16
        bt = BlockTable(pool)
        ids = [bt.allocate_block() for _ in range(pool)]
        rng.shuffle(ids)
        for i in ids:
            bt.free_block(i)
        heads = [bt.allocate_chain(-(-n // 64)) for n in lens]
        max_b = max(-(-n // 64) for n in lens)
        pt = torch.from_numpy(bt.export_page_table(heads, max_b)).to(device)
        g = torch.Generator(device=device).manual_seed(2)
        qkv = [(torch.randn(pool, H, 64, D, generator=g, device=device) * c["std"]).to(dt)
               for _ in range(3)]
        half = D // 2
        inv = 1.0 / (c["rope_base"] ** (torch.arange(half, dtype=torch.float64) * 2.0 / D))
        ang = torch.arange(max_b * 64, dtype=torch.float64)[:, None] * inv[None, :]
        cos, sin = torch.cos(ang).float().to(device), torch.sin(ang).float().to(device)
        lens_t = torch.tensor(lens, dtype=torch.int32, device=device)
        call_args = (pt, *qkv, lens_t, cos, sin)
        flops = 4.0 * H * D * sum(n * n for n in lens)
        res = {"shape": dict(c, lens=None if "ctx_min" in c else lens)}
        outs = {}
        for side, fn in (("reference_triton", ref.block_attention), ("ours", block_attention)):
            try:
                for _ in range(2):
                    o = fn(*call_args)
                torch.cuda.synchronize(device)
                steps = 5
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(steps):
                    o = fn(*call_args)
                e1.record()
                torch.cuda.synchronize(device)
                ms = e0.elapsed_time(e1) / steps
                res[side] = {"ms_per_call": ms, "TFLOP/s": flops / (ms / 1000.0) / 1e12}
                outs[side] = o
            except Exception as exc:  # noqa: BLE001 - record why a side could not run
                res[side] = {"error": f"{type(exc).__name__}: {str(exc)[:300]}"}
        if len(outs) == 2:
            errs = torch.cat([(outs["ours"][s, :, :n].float() - outs["reference_triton"][s, :, :n]
                               .float()).abs().reshape(-1) for s, n in enumerate(lens)])
            res["max_abs_diff"], res["mean_abs_diff"] = float(errs.max()), float(errs.mean())
            res["speedup_vs_reference"] = (res["reference_triton"]["ms_per_call"] /
                                           res["ours"]["ms_per_call"])
        out[name] = res
        del qkv, outs
        torch.cuda.empty_cache()
    return out


def run_reference_kernel(args):
    world, rank, local = _dist_env()
    device = _init_dist(world, local)
    if rank == 0:
        line = {"metric": "full self-attention per call: the reference's Triton kernel vs ours",
                "n_gpus": 1, "data": "synthetic", **_reference_kernel_leg(args, device)}
        print(json.dumps(line), flush=True)
    return 0


SCOPED = dict(workload="mha_paged_decode_fp16_scoped", seqs=32, heads=32, head_dim=128,
              dtype="fp16", ctx_min=512, ctx_max=4096, pool_blocks=4096, rope_base=10000.0,
              segment_min=32, segment_max=512, seed=2)


def run_decode_scoped(args):
    """Scoped MHA decode (fp16, 32 sequences, lens U[512, 4096], 4096-block pool, Table-1
    scope from random segments: the first GLOBAL, later ones LOCAL with p = 1/2).

    Times the scoped decode, then the same batch unscoped. A block with no allowed key for
    the query is never loaded, so the scoped step reads only the blocks its scopes reach:
    ``bytes_needed`` counts those, ``bytes_all_keys`` every cached key.
    """
    import numpy as np
    import torch

    from oracle import attention_oracle as ao  # RoPE tables and the spot check
    from src.block_table import BlockTable
    from src.engine import random_segments
    from src.kernels.block_attention import DecodeCall
    from src.scoping_mask import decode_scope

    P = SCOPED
    device = torch.device("cuda", 0)
    rng = random.Random(P["seed"])
    S, H, D = P["seqs"], P["heads"], P["head_dim"]
    lens = [rng.randint(P["ctx_min"], P["ctx_max"]) for _ in range(S)]
    bt = BlockTable(P["pool_blocks"])
    ids = [bt.allocate_block() for _ in range(P["pool_blocks"])]
    rng.shuffle(ids)
    for i in ids:
        bt.free_block(i)
    heads = [bt.allocate_chain(-(-n // 64)) for n in lens]
    pt = torch.from_numpy(bt.export_page_table(heads, -(-P["ctx_max"] // 64))).to(device)
    g = torch.Generator(device=device).manual_seed(P["seed"])
    k = (torch.randn(P["pool_blocks"], H, 64, D, generator=g, device=device) * 0.5).half()
    v = (torch.randn(P["pool_blocks"], H, 64, D, generator=g, device=device) * 0.5).half()
    q = (torch.randn(S, H, D, generator=g, device=device) * 0.5).half()
    cos, sin = ao.rope_tables(P["ctx_max"], D, P["rope_base"])
    cos_d, sin_d = torch.from_numpy(cos).to(device), torch.from_numpy(sin).to(device)
    W = -(-P["ctx_max"] // 16) * 16
    tags = np.zeros((S, W), np.uint8)
    span = np.zeros((S, 2), np.int32)
    needed_tok = 0
    for s, n in enumerate(lens):
        t, lo, hi = decode_scope(random_segments(rng, n, P["segment_min"], P["segment_max"]), n - 1)
        tags[s, :n] = t
        span[s] = (lo, hi)
        for b in range(-(-n // 64)):
            a, e = b * 64, min(n, b * 64 + 64)
            if t[a:e].any() or (a < hi and e > lo):
                needed_tok += e - a
    lens_d = torch.tensor(lens, dtype=torch.int32, device=device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    scope = (torch.from_numpy(tags).to(device), torch.from_numpy(span).to(device))
    calls = {"scoped": DecodeCall(pt, q, k, v, lens_d, cos_d, sin_d, scope=scope, status=status),
             "unscoped": DecodeCall(pt, q, k, v, lens_d, cos_d, sin_d, status=status)}
    per_tok = H * D * 2 * 2
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    res = {}
    for name, call in calls.items():
        for _ in range(max(args.warmup, 3)):
            call.launch()
        torch.cuda.synchronize()
        total = 0.0
        for _ in range(args.steps):
            flush.zero_()  # the batch (1.2 GB) exceeds L2 anyway; flushed so no step starts warm
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            call.launch()
            e1.record()
            torch.cuda.synchronize()
            total += e0.elapsed_time(e1)
        res[name] = total / args.steps
    out = calls["scoped"].out
    want = ao.decode_attention(pt[:4].cpu().numpy(), q[:4].float().cpu().numpy(),
                               k.float().cpu().numpy(), v.float().cpu().numpy(), lens[:4], cos,
                               sin, scope_tags=tags[:4], scope_span=span[:4])
    err = np.abs(out[:4].float().cpu().numpy() - want)
    hbm, src = _peaks()
    ms = res["scoped"]
    gbs = needed_tok * per_tok / (ms / 1000.0) / 1e9
    line = {
        "metric": "scoped MHA paged-decode tokens/s (fp16, Table-1 scope)", "value": S / (ms / 1000.0),
        "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "dtype": "fp16",
        "data": "synthetic (seeded; random K/V/Q and segments)", "config": P,
        "bytes_all_keys": sum(lens) * per_tok, "bytes_needed": needed_tok * per_tok,
        "unscoped_ms_per_step": res["unscoped"],
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                     "frac": gbs / hbm, "peak_source": src,
                     "note": "bytes of the blocks the scopes reach / scoped step time"},
        "check": {"rows": 4, "max_abs": float(err.max()), "mean_abs": float(err.mean()),
                  "kernel_status": int(status.item())},
    }
    print(json.dumps(line), flush=True)
    return 0


SERVING = dict(workload="serving_trace_llama3_8b_attention", requests=512, rate_per_s=64.0,
               prompt_median=2048, prompt_sigma=1.0, prompt_min=128, prompt_max=16384,
               output_tokens=256, q_heads=32, kv_heads=8, head_dim=128, hidden=4096, dtype="bf16",
               rope_base=500000.0, chunk=2048, prefill_tokens_per_step=8192,
               pool_fraction=0.25, seed=17)


def _serving_measure(args, world: int, rank: int, device, rate: float):
    """The serving trace: Poisson arrivals at ``rate`` per second, lognormal prompts, 256
    output tokens each, continuous batching through the native allocator, token scopes
    from random segments.

    Every rank builds the same seeded trace; the Supervisor's placement (LPT on total
    tokens, ``src.engine.shard_requests``) gives each rank whole requests, served by that
    GPU's engine (sequence-sharded KV; no collective on the data path). value = all ranks'
    output tokens / the slowest rank's wall time. At the stated 64 requests/s the trace's
    own ~8 s of arrivals bound it; a compressed rate (all 512 requests within a fraction
    of a second) measures the engine.
    """
    import torch
    import torch.distributed as dist

    from src.engine import Engine, StandInBackend, make_trace, shard_requests
    from src.serving import KVPool

    P = SERVING
    trace = make_trace(P["requests"], rate, P["prompt_median"], P["prompt_sigma"],
                       P["prompt_min"], P["prompt_max"], P["output_tokens"], P["seed"])
    mine = shard_requests(trace, world)[rank]
    max_total = P["prompt_max"] + P["output_tokens"]
    blocks = sum(r.blocks for r in mine)
    pool_blocks = max(-(-max_total // 64) + 1, int(blocks * P["pool_fraction"]))
    pool = KVPool(device=device, num_blocks=pool_blocks, kv_heads=P["kv_heads"],
                  head_dim=P["head_dim"], dtype=torch.bfloat16, max_positions=max_total,
                  rope_base=P["rope_base"])
    be = StandInBackend(pool, P["q_heads"], hidden=P["hidden"], max_total=max_total,
                        slots=1024, seed=rank)
    # warm-up: a short trace of its own through the same pool (all chains freed after)
    warm = make_trace(8, 1000.0, 600, 0.5, 128, 2048, 8, seed=1000 + rank)
    Engine(pool.table, be, chunk=P["chunk"], prefill_tokens=P["prefill_tokens_per_step"]).run(warm)
    torch.cuda.synchronize(device)
    be.kv_bytes = 0
    be.attn_events = {"prefill": [], "decode": []}
    eng = Engine(pool.table, be, chunk=P["chunk"], prefill_tokens=P["prefill_tokens_per_step"],
                 slots=1024)
    if world > 1:
        dist.barrier()
    class _DeviceTimer:
        """Token times from CUDA events recorded after each step (no per-step sync)."""

        def start(self):
            self.e0 = torch.cuda.Event(enable_timing=True)
            self.e0.record()

        def mark(self):
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            return ev

        def sync(self):
            torch.cuda.synchronize(device)

        def seconds(self, ev):
            return self.e0.elapsed_time(ev) / 1000.0

    with ClockSampler(device.index) as clk:
        # the host runs ahead of the device; token times are the device completion times of
        # the steps that produced them (events), read once at the end
        st = eng.run(mine, timer=_DeviceTimer())
        torch.cuda.synchronize(device)
    dec_ms, pre_ms = be.attn_ms("decode"), be.attn_ms("prefill")
    vals = torch.tensor([st["generated_tokens"], st["wall_s"], be.kv_bytes, dec_ms],
                        dtype=torch.float64, device=device)
    if world > 1:
        tot = vals.clone()
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
        mx = vals.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        gen, wall, kv_total = float(tot[0]), float(mx[1]), float(tot[2])
    else:
        gen, wall, kv_total = float(vals[0]), float(vals[1]), float(vals[2])
    peak = None
    pk = ROOT / "MEASURED_PEAKS.json"
    if pk.exists():
        peak = float(json.loads(pk.read_text())["hbm_gbs"])
    dec_gbs = be.kv_bytes / (dec_ms / 1000.0) / 1e9 if dec_ms > 0 else None
    arrivals_s = max(r.arrival for r in trace)
    kv_rank0 = be.kv_bytes
    del eng, be, pool
    torch.cuda.empty_cache()
    return {
        "metric": "serving trace output tokens/s (512 requests, Poisson arrivals, 256 output "
                  "tokens)",
        "value": gen / wall, "unit": "tokens/s", "n_gpus": world, "higher_is_better": True,
        "scaling": "strong", "dtype": "bf16",
        "data": "synthetic (seeded trace; random-init stand-in projections, no dataset)",
        "config": dict(P, rate_per_s=rate, parallelism=f"dp{world} (whole requests per GPU, "
                                                       "LPT)", pool_blocks_rank0=pool_blocks,
                       last_arrival_s=arrivals_s),
        "wall_s": wall, "generated_tokens": gen,
        "arrival_bound": bool(arrivals_s > 0.5 * wall),
        "rank0": {"requests": st["requests"], "steps": st["steps"], "ttft_s": st["ttft_s"],
                  "tpot_s": st["tpot_s"], "peak_running": st["peak_running"],
                  "peak_blocks": st["peak_blocks"], "prompt_tokens": st["prompt_tokens"],
                  "prefill_attention_ms": pre_ms},
        "decode_attention": {"timing": "CUDA events around each decode call (decode kernels "
                                       "and the host gap between their launches)",
                             "bytes_rank0": kv_rank0, "ms_rank0": dec_ms,
                             "GB/s_rank0": dec_gbs, "peak_GB/s": peak,
                             "frac": (dec_gbs / peak) if (dec_gbs and peak) else None,
                             "bytes_all_ranks": kv_total},
        "clocks": clk.summary(),
    }


def _serving_leg(args, world: int, rank: int, device):
    """The serving trace at a compressed arrival rate, as a sub-object of the headline line."""
    line = _serving_measure(args, world, rank, device, args.serving_rate)
    return {k: line[k] for k in ("metric", "value", "unit", "scaling", "wall_s",
                                 "generated_tokens", "arrival_bound", "rank0",
                                 "decode_attention", "config")}


def run_serving(args):
    import torch.distributed as dist

    world, rank, local = _dist_env()
    device = _init_dist(world, local, timeout_s=300)
    line = _serving_measure(args, world, rank, device,
                            args.serving_rate if args.serving_rate > 0 else SERVING["rate_per_s"])
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--split-blocks", type=int, default=0)
    ap.add_argument("--kernel", default="auto", choices=["auto", "tc", "tc2", "streamk", "simt"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--no-prefill", action="store_true",
                    help="skip the chunked-prefill sub-object of the decode line")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="how the Supervisor's step moves queries and rows between GPUs "
                         "(N > 1): peer memory over NVLink, or NCCL point-to-point")
    ap.add_argument("--serving-rate", type=float, default=0.0,
                    help="arrivals per second of the serving trace (--workload serving: the "
                         "stated 64; the headline line's serving leg: 4096, all 512 requests "
                         "within ~0.13 s, so the engine, not the arrivals, sets the time)")
    ap.add_argument("--no-serving", action="store_true",
                    help="skip the serving-trace sub-object of the decode line")
    ap.add_argument("--no-supervisor-api", action="store_true",
                    help="skip the Supervisor.decode_step sub-measurement (N = 1)")
    ap.add_argument("--no-reference-kernel", action="store_true",
                    help="skip the reference Triton kernel comparison (N = 1 only)")
    ap.add_argument("--prefill-steps", type=int, default=0,
                    help="timed prefill passes (default: --steps)")
    ap.add_argument("--workload", choices=["decode", "prefill", "serving", "decode-scoped",
                                           "reference-kernel"],
                    default="decode",
                    help="decode (the headline metric), the chunked-prefill tensor-core pass, "
                         "the serving trace (continuous batching end to end) or the scoped "
                         "MHA decode")
    ap.add_argument("--seqs", type=int, default=0,
                    help="sequences per GPU (default: the workload's 256); smaller values "
                         "make a profiling case of the same kernel")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "prefill":
        return run_prefill(args)
    if args.workload == "serving":
        return run_serving(args)
    if args.workload == "decode-scoped":
        return run_decode_scoped(args)
    if args.workload == "reference-kernel":
        return run_reference_kernel(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
