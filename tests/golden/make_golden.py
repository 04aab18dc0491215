"""Regenerates the golden fixtures in this folder by running the REFERENCE.

Run in a container where the reference checkout is mounted:

    python tests/golden/make_golden.py --reference <reference checkout>

(or set OURO_REFERENCE; the script stops with a message when neither names a
checkout holding src/kernels/block_attention.py).

It imports the reference's own ``src`` package (BlockTable, dense_reference,
golden_attention_mt, block_sparse_mask) and records, for seeded inputs built
by ``cases.py``:

* ``attn_small.npz``   dense_reference on the reference GPU-test shape
                       (fp32 with bias + block mask, fp32 plain, fp16)
* ``decode_c1.npz``    config-1 decode rows (and a few full rows) of
                       dense_reference, plus the reference allocator's page table
* ``decode_c2s.npz``   two fp16 MHA sequences of the config-2 shape with a
                       Table-1 scope mask passed to dense_reference as a -inf bias
* ``decode_gqa.npz``   a GQA (group 8) bf16 decode case via K/V repeat_interleave
* ``golden_mt.npz``    golden_attention_mt (pure-Python oracle) outputs with
                       their fp32-rounded payloads, d_head 8 and 32
* ``alloc_scripts.json`` op-by-op results of the reference Python BlockTable
* ``scope_masks.json`` block_sparse_mask for seeded span sets

Only this script needs the reference checkout; the tests read the recorded files.
"""

from __future__ import annotations

import argparse
import os
import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def _load_reference(ref: Path):
    sys.path.insert(0, str(ref))
    sys.path.insert(0, str(HERE))
    import cases  # noqa: E402
    from src import block_table as rbt  # noqa: E402  (the reference's package)
    from src import scoping_mask as rsm  # noqa: E402
    from src.kernels import block_attention as rba  # noqa: E402
    from src.kernels import reference_attention as rra  # noqa: E402

    assert Path(rbt.__file__).resolve().is_relative_to(ref.resolve()), rbt.__file__
    return cases, rbt, rsm, rba, rra


def gen_attn_small(torch, np, cases, rbt, rba):
    out = {}
    specs = [("bm", 1234, torch.float32, True), ("plain", 77, torch.float32, False),
             ("f16", 5, torch.float16, False)]
    for name, seed, dtype, with_bm in specs:
        c = cases.small_full_case(torch, rbt.BlockTable, seed, dtype=dtype)
        pt = torch.tensor(c["rows"], dtype=torch.int32)
        kw = {}
        if with_bm:
            gen = torch.Generator().manual_seed(seed + 1)
            maxlen = max(c["lens"])
            bias = torch.randn(1, 2, maxlen, maxlen, generator=gen) * 0.25
            scope = torch.randint(0, 2, (2, 3, 3), generator=gen)
            scope |= torch.eye(3, dtype=torch.int64)
            kw = dict(bias=bias, mask=scope.to(torch.int8))
            out[f"{name}_biassum"] = np.asarray(cases.input_checksum(bias))
            out[f"{name}_mask"] = scope.to(torch.int8).numpy()
        ref = rba.dense_reference(pt, c["q_cache"], c["k_cache"], c["v_cache"], c["lens"],
                                  c["cos"], c["sin"], **kw)
        out[f"{name}_out"] = ref.numpy()
        out[f"{name}_rows"] = np.asarray(c["rows"], dtype=np.int32)
        out[f"{name}_lens"] = np.asarray(c["lens"], dtype=np.int32)
        out[f"{name}_qsum"] = np.asarray(cases.input_checksum(c["q_cache"]))
    np.savez_compressed(HERE / "attn_small.npz", **out)


def gen_decode_c1(torch, np, cases, rbt, rba):
    c = cases.config1_case(torch, rbt.BlockTable, seed=1)
    pt = torch.tensor(c["rows"], dtype=torch.int32)
    ref = rba.dense_reference(pt, c["q_cache"], c["k_cache"], c["v_cache"], c["lens"],
                              c["cos"], c["sin"])
    lens = c["lens"]
    dec = np.stack([ref[s, :, lens[s] - 1, :].numpy() for s in range(len(lens))])
    probe_rows = [0, 63, 129]  # rows also checked through the full-attention path
    probes = np.stack([ref[3, :, r, :].numpy() for r in probe_rows])
    np.savez_compressed(
        HERE / "decode_c1.npz", decode=dec, probes=probes, probe_rows=np.asarray(probe_rows),
        rows=np.asarray(c["rows"], dtype=np.int32), lens=np.asarray(lens, dtype=np.int32),
        qsum=np.asarray(cases.input_checksum(c["q_cache"])),
        ksum=np.asarray(cases.input_checksum(c["k_cache"])))


def gen_decode_c2s(torch, np, cases, rbt, rsm, rba):
    c = cases.config2_slice_case(torch, rbt.BlockTable)
    lens = c["lens"]
    S, maxlen = len(lens), max(lens)
    bias = torch.full((S, 1, maxlen, maxlen), float("-inf"))
    for s, spans in enumerate(c["spans"]):
        m = torch.tensor(rsm.block_sparse_mask(spans), dtype=torch.bool)
        T = lens[s]
        bias[s, 0, :T, :T] = torch.where(m, 0.0, float("-inf"))
    pt = torch.tensor(c["rows"], dtype=torch.int32)
    ref = rba.dense_reference(pt, c["q_cache"], c["k_cache"], c["v_cache"], lens,
                              c["cos"], c["sin"], bias=bias)
    dec = np.stack([ref[s, :, lens[s] - 1, :].numpy() for s in range(S)])
    np.savez_compressed(
        HERE / "decode_c2s.npz", decode=dec, rows=np.asarray(c["rows"], dtype=np.int32),
        lens=np.asarray(lens, dtype=np.int32),
        spans=np.asarray(json.dumps(c["spans"])),
        qsum=np.asarray(cases.input_checksum(c["q_cache"])))


def gen_decode_gqa(torch, np, cases, rbt, rba):
    c = cases.gqa_decode_case(torch, rbt.BlockTable)
    lens, hq, hkv = c["lens"], c["q"].shape[1], c["k_cache"].shape[1]
    grp = hq // hkv
    k = c["k_cache"].float().repeat_interleave(grp, dim=1)
    v = c["v_cache"].float().repeat_interleave(grp, dim=1)
    qc = torch.zeros_like(k)
    for s, T in enumerate(lens):
        last = c["rows"][s][(T - 1) // 64]
        qc[last, :, (T - 1) % 64, :] = c["q"][s].float()
    pt = torch.tensor(c["rows"], dtype=torch.int32)
    ref = rba.dense_reference(pt, qc, k, v, lens, c["cos"], c["sin"])
    dec = np.stack([ref[s, :, lens[s] - 1, :].numpy() for s in range(len(lens))])
    np.savez_compressed(
        HERE / "decode_gqa.npz", decode=dec, rows=np.asarray(c["rows"], dtype=np.int32),
        lens=np.asarray(lens, dtype=np.int32), qsum=np.asarray(cases.input_checksum(c["q"])))


def gen_golden_mt(np, rbt, rra):
    out = {}
    for d in (8, 32):
        bt = rbt.BlockTable(max_blocks=16)
        heads = [bt.allocate_chain(3), bt.allocate_chain(2)]
        blocks = rra.build_multi_token_payloads(bt, heads, d, seed=f"golden-{d}")
        ids = sorted(blocks)
        pay = np.zeros((len(ids), 3, 64, d), dtype=np.float32)
        for bi, pid in enumerate(ids):
            for ci, comp in enumerate("qkv"):
                pay[bi, ci] = np.asarray(blocks[pid][comp], dtype=np.float32)
        # feed the fp32-rounded payloads back so the golden is exact for them
        rounded = {pid: {comp: pay[bi, ci].astype(np.float64).tolist()
                         for ci, comp in enumerate("qkv")} for bi, pid in enumerate(ids)}
        rows = [list(bt.walk(h)) for h in heads]
        lens = [150, 128]
        half = d // 2
        inv = [10000.0 ** (-2.0 * t / d) for t in range(half)]
        cos_t = np.asarray([[np.cos(p * w) for w in inv] for p in range(256)], dtype=np.float32)
        sin_t = np.asarray([[np.sin(p * w) for w in inv] for p in range(256)], dtype=np.float32)
        qpos = [[149, 0, 77], [127, 64]]
        gold = rra.golden_attention_mt(rows, rounded, lens, cos_t.astype(np.float64).tolist(),
                                       sin_t.astype(np.float64).tolist(),
                                       query_positions=qpos)
        out[f"d{d}_payload"] = pay
        out[f"d{d}_ids"] = np.asarray(ids, dtype=np.int32)
        out[f"d{d}_rows"] = np.asarray([r + [-1] * (3 - len(r)) for r in rows], dtype=np.int32)
        out[f"d{d}_lens"] = np.asarray(lens, dtype=np.int32)
        out[f"d{d}_qpos"] = np.asarray(json.dumps(qpos))
        out[f"d{d}_gold"] = np.asarray(gold, dtype=np.float64)
    np.savez_compressed(HERE / "golden_mt.npz", **out)


def gen_alloc_scripts(cases, rbt):
    scripts = []
    for seed in (1, 2, 3, 42, 7, 99):
        mb = 24 if seed != 99 else 8
        bt = rbt.BlockTable(max_blocks=mb)
        steps = []
        for op in cases.alloc_script(seed, max_blocks=mb):
            kind = op[0]
            if kind == "link":
                allocated = {i for i in range(mb) if bt.blocks[i] is not None}
                if not cases.link_is_safe(lambda i: bt.next_ptr[i], allocated, op[1], op[2]):
                    steps.append({"op": op, "skip": True})
                    continue
            try:
                if kind == "alloc":
                    res = bt.allocate_block()
                elif kind == "free":
                    res = bt.free_block(op[1])
                elif kind == "chain":
                    res = bt.allocate_chain(op[1])
                elif kind == "expand":
                    res = bt.expand_chain(op[1])
                elif kind == "link":
                    res = bt.link(op[1], op[2])
                elif kind == "walk":
                    res = list(bt.walk(op[1]))
                elif kind == "len":
                    res = bt.chain_len(op[1])
                elif kind == "resolve":
                    res = bt.resolve_block(op[1], op[2])
                elif kind == "row":
                    res = bt.page_table_row(op[1], pad_to=op[2])
                elif kind == "cell":
                    bt.get_block(op[1])[op[2]] = op[3]
                    res = bt.get_block(op[1])[op[2]]
                else:
                    raise AssertionError(kind)
                steps.append({"op": op, "result": res})
            except RuntimeError as exc:
                steps.append({"op": op, "error": str(exc)})
        final = {
            "num_free": bt.num_free,
            "next_ptr": [bt.next_ptr[i] if bt.blocks[i] is not None else -1 for i in range(mb)],
            "payload": [None if b is None else list(b) for b in bt.blocks],
            "free_list": list(bt.free_list),
        }
        scripts.append({"seed": seed, "max_blocks": mb, "steps": steps, "final": final})
    (HERE / "alloc_scripts.json").write_text(json.dumps(scripts, separators=(",", ":")))


def gen_scope_masks(cases, rsm):
    import random
    out = []
    for seed in range(12):
        rng = random.Random(seed)
        L = rng.randint(1, 40)
        spans = cases.segment_spans(L, seed, lo=1, hi=9, p_local=0.6)
        mask = rsm.block_sparse_mask(spans)
        out.append({"spans": spans, "mask": ["".join("1" if v else "0" for v in r) for r in mask]})
    (HERE / "scope_masks.json").write_text(json.dumps(out, separators=(",", ":")))


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("OURO_REFERENCE"),
                    help="the reference checkout (default: $OURO_REFERENCE)")
    args = ap.parse_args()
    if not args.reference or not (Path(args.reference) / "src" / "kernels" /
                                  "block_attention.py").exists():
        ap.error("pass --reference <reference checkout> or set OURO_REFERENCE")
    import numpy as np
    import torch

    torch.set_num_threads(8)
    cases, rbt, rsm, rba, rra = _load_reference(Path(args.reference))
    gen_alloc_scripts(cases, rbt)
    gen_scope_masks(cases, rsm)
    gen_golden_mt(np, rbt, rra)
    gen_attn_small(torch, np, cases, rbt, rba)
    gen_decode_c1(torch, np, cases, rbt, rba)
    gen_decode_gqa(torch, np, cases, rbt, rba)
    gen_decode_c2s(torch, np, cases, rbt, rsm, rba)
    for p in sorted(HERE.glob("*.npz")) + sorted(HERE.glob("*.json")):
        print(f"{p.name}: {p.stat().st_size} bytes")
    return 0


if __name__ == "__main__":
    sys.exit(main())
