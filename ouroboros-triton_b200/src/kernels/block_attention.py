"""Paged block attention on B200: the drop-in for the reference module
``src/kernels/block_attention.py``.

Entry points
  * :func:`block_attention` — the reference's entry point, same signature and
    result: full self-attention over every row of every sequence, paged
    q/k/v, RoPE, additive bias, block mask (block_attention.py:368-527).
  * :func:`chunked_prefill_attention` — a dense chunk of query rows per
    sequence over all its earlier keys, causal, GQA.
  * :func:`block_attention_decode` — one query token per sequence (the decode
    step) over its paged K/V: GQA, explicit positions, split-K, fused RoPE,
    block mask and token-granular Table-1 scope. sm_100a kernels in
    ``csrc/decode_tc.cu`` (tensor cores) and ``csrc/decode_simt.cu``.
  * :func:`validate_bias_shape`, :func:`validate_mask_shape`,
    :func:`_broadcast_strides` — the reference's pure-Python helpers
    (block_attention.py:90-178), same rules and messages.

Every launcher calls the native library through its C ABI
(``include/ouroboros_b200.h``). There is no Triton and no CPU path: without a
CUDA device, or without the built library, calls raise RuntimeError.
"""

from __future__ import annotations

import ctypes
from typing import Sequence

try:  # import safety, as in the reference (block_attention.py:55-71)
    import torch

    HAS_TORCH = True
except ImportError:  # pragma: no cover
    torch = None  # type: ignore[assignment]
    HAS_TORCH = False

from .. import _native
from ..block_table import BLOCK_SIZE, PAD_ID
from . import _capi

#: The reference's flag for its Triton backend. This implementation never uses
#: Triton; the flag stays for import compatibility and is always False.
HAS_TRITON = False

__all__ = [
    "HAS_TRITON",
    "HAS_TORCH",
    "block_attention",
    "block_attention_decode",
    "chunked_prefill_attention",
    "paged_kv_append",
    "decode_plan",
    "validate_bias_shape",
    "validate_mask_shape",
    "validate_page_table",
]

_KERNELS = {"auto": 0, "simt": 1, "cuda_cores": 1, "tensor_cores": 2, "tc": 2, "tc2": 3,
            "streamk": 4}


# ---------------------------------------------------------------------------
# Shape helpers (reference block_attention.py:90-178)
# ---------------------------------------------------------------------------


def validate_bias_shape(bias_shape: Sequence[int], *, num_heads: int, q_len: int, kv_len: int,
                        num_seqs: int | None = None) -> None:
    """Bias must broadcast to [S, H, Q, K] (right-aligned, dims equal or 1)."""
    shape = tuple(int(d) for d in bias_shape)
    targets = (num_seqs if num_seqs is not None else 1, num_heads, q_len, kv_len)
    if len(shape) > 4:
        raise RuntimeError(f"bias rank {len(shape)} > 4, cannot broadcast to [S, H, Q, K]")
    padded = (1,) * (4 - len(shape)) + shape
    for got, want in zip(padded, targets):
        if got != 1 and got != want:
            raise RuntimeError(
                f"bias dim {got} incompatible with expected {want} "
                f"(shape {shape} vs [S={targets[0]}, H={num_heads}, Q={q_len}, K={kv_len}])")


def validate_mask_shape(mask_shape: Sequence[int], *, num_q_blocks: int, num_kv_blocks: int,
                        num_seqs: int | None = None) -> None:
    """Block mask must broadcast to [S, QB, KB]; a rank-1 mask is per KV block."""
    shape = tuple(int(d) for d in mask_shape)
    targets = (num_seqs if num_seqs is not None else 1, num_q_blocks, num_kv_blocks)
    if len(shape) > 3:
        raise RuntimeError(f"mask rank {len(shape)} > 3, cannot broadcast to [S, QB, KB]")
    padded = (1, 1, shape[0]) if len(shape) == 1 else (1,) * (3 - len(shape)) + shape
    for got, want in zip(padded, targets):
        if got != 1 and got != want:
            raise RuntimeError(
                f"mask dim {got} incompatible with expected {want} "
                f"(shape {shape} vs [S={targets[0]}, QB={num_q_blocks}, KB={num_kv_blocks}])")


def _broadcast_strides(shape: Sequence[int], target: Sequence[int]) -> tuple[int, ...]:
    """Element strides of a contiguous ``shape`` viewed under ``target``; broadcast axes get 0."""
    shape = tuple(int(d) for d in shape)
    if len(shape) > len(target):
        raise RuntimeError(f"rank {len(shape)} exceeds target rank {len(target)}")
    padded = (1,) * (len(target) - len(shape)) + shape
    for got, want in zip(padded, target):
        if got != 1 and got != want:
            raise RuntimeError(f"dim {got} incompatible with {want}")
    strides, running = [], 1
    for ax in range(len(target) - 1, -1, -1):
        strides.append(0 if padded[ax] == 1 else running)
        running *= padded[ax]
    return tuple(reversed(strides))


# ---------------------------------------------------------------------------
# Device plumbing
# ---------------------------------------------------------------------------


def _require_cuda() -> None:
    if not HAS_TORCH:
        raise RuntimeError("block attention requires torch (not installed on this host)")
    if not torch.cuda.is_available():
        raise RuntimeError("block_attention requires a CUDA device")
    _native.lib()  # raises if the native library is not built


def _dtype_code(dt) -> int:
    if dt == torch.float32:
        return _native.DTYPE_F32
    if dt == torch.float16:
        return _native.DTYPE_F16
    if dt == torch.bfloat16:
        return _native.DTYPE_BF16
    raise RuntimeError(f"unsupported cache dtype {dt}; want float32, float16 or bfloat16")


def _device_of(*tensors):
    for t in tensors:
        if t is not None and hasattr(t, "is_cuda") and t.is_cuda:
            return t.device
    return torch.device("cuda", torch.cuda.current_device())


def _on(t, device, dtype=None):
    """``t`` as a contiguous tensor on ``device`` (converted from lists/ints if needed)."""
    if t is None:
        return None
    if not torch.is_tensor(t):
        t = torch.as_tensor(t)
    t = t.to(device=device, dtype=dtype if dtype is not None else t.dtype, non_blocking=True)
    return t.contiguous()


def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _stream_handle(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def validate_page_table(page_table, seq_lens, num_phys_blocks: int) -> None:
    """Raises RuntimeError on the first bad page-table entry.

    The reference checks every entry on the host after ``.tolist()``
    (block_attention.py:445-466); here one device pass finds the lowest bad
    entry and 8 bytes come back. Same message texts.
    """
    _validate_page_table(page_table, seq_lens, num_phys_blocks)


def _validate_page_table(page_table, seq_lens, num_phys_blocks: int, with_max_len=False):
    """validate_page_table; with ``with_max_len`` also returns max(seq_lens), read back
    in the same transfer as the check's verdict (one synchronisation per call)."""
    _require_cuda()
    S, max_b = page_table.shape
    device = page_table.device
    report = torch.empty(2, dtype=torch.int64, device=device)
    _native.check(_native.lib().ouro_validate_page_table(
        _ptr(page_table), _ptr(seq_lens), S, max_b, int(num_phys_blocks), _ptr(report),
        _stream_handle(device)), "validate_page_table")
    if with_max_len:
        if S:
            report[1:].copy_(seq_lens.max().reshape(1))
        else:
            report[1:].zero_()
        key, max_len = report.tolist()
    else:
        key, max_len = int(report[0].item()), 0
    key &= 0xFFFFFFFFFFFFFFFF
    if key == 0xFFFFFFFFFFFFFFFF:
        return max_len
    idx, code = key >> 2, key & 3
    s, n = divmod(idx, max_b) if max_b else (idx, 0)
    if code == 3:
        ln = int(seq_lens[s].item())
        need = -(-ln // BLOCK_SIZE)
        if ln < 0:
            raise RuntimeError(f"sequence {s} has negative length {ln}")
        raise RuntimeError(f"sequence {s} needs {need} blocks > table width {max_b}")
    phys = int(page_table[s, n].item())
    if code == 2:
        ln = int(seq_lens[s].item())
        raise RuntimeError(
            f"page_table[{s}][{n}] must be PAD_ID({PAD_ID}) beyond seq_len {ln}, got {phys}")
    raise RuntimeError(
        f"page_table[{s}][{n}]={phys} out of range for {num_phys_blocks} physical blocks")


_SM_SCOPE_ALIGN = 16


def _scope_tensors(scope, S: int, device):
    """(tags [S, W] uint8 with W % 16 == 0, span [S, 2] int32) from ``scope``.

    ``scope`` is ``(tags, span)``: tags [S, L] (bool / uint8, 1 = GLOBAL token)
    and span [S, 2] (the query's LOCAL span, (0, 0) for a GLOBAL query).
    """
    tags, span = scope
    tags = torch.as_tensor(tags)
    if tags.dim() != 2 or tags.shape[0] != S:
        raise RuntimeError(f"scope tags must be [S={S}, L], got {tuple(tags.shape)}")
    L = tags.shape[1]
    if (tags.dtype == torch.uint8 and tags.device == torch.device(device) and L > 0
            and L % _SM_SCOPE_ALIGN == 0 and tags.is_contiguous()
            and tags.data_ptr() % _SM_SCOPE_ALIGN == 0):
        padded = tags  # already in the kernel's layout: used in place
    else:
        W = max(_SM_SCOPE_ALIGN, -(-L // _SM_SCOPE_ALIGN) * _SM_SCOPE_ALIGN)
        padded = torch.zeros((S, W), dtype=torch.uint8, device=device)
        padded[:, :L] = tags.to(device=device, dtype=torch.uint8)
    span = _on(span, device, torch.int32)
    if span is None or tuple(span.shape) != (S, 2):
        raise RuntimeError(f"scope span must be [S={S}, 2]")
    return padded, span


def _decode_args(page_table, q, k_cache, v_cache, seq_lens, cos, sin, positions, mask, scope,
                 causal, softmax_scale, split_blocks, kernel, out, workspace, status,
                 total_blocks=0, max_seq_blocks=0):
    S, Hq, D = q.shape
    n_phys, Hkv, blk, Dk = k_cache.shape
    a = _capi.DecodeArgs()
    a.q, a.k_cache, a.v_cache = _ptr(q), _ptr(k_cache), _ptr(v_cache)
    a.page_table, a.seq_lens = _ptr(page_table), _ptr(seq_lens)
    a.positions = _ptr(positions)
    a.cos, a.sin = _ptr(cos), _ptr(sin)
    if mask is not None:
        a.block_mask = _ptr(mask[0])
        a.mask_stride_s, a.mask_stride_q, a.mask_stride_k = mask[1]
    if scope is not None:
        a.scope_tags = _ptr(scope[0])
        a.scope_stride = scope[0].shape[1]
        a.scope_span = _ptr(scope[1])
    a.out = _ptr(out)
    if workspace is not None:
        a.workspace = _ptr(workspace)
        a.workspace_bytes = workspace.numel() * workspace.element_size()
    a.status = _ptr(status)
    a.num_seqs, a.num_q_heads, a.num_kv_heads, a.head_dim = S, Hq, Hkv, D
    a.max_blocks = page_table.shape[1]
    a.num_phys_blocks = n_phys
    a.max_positions = cos.shape[0]
    a.dtype = _dtype_code(k_cache.dtype)
    a.split_blocks = int(split_blocks)
    a.causal = 1 if causal else 0
    a.kernel = _KERNELS[kernel]
    a.softmax_scale = float(softmax_scale) if softmax_scale is not None else 0.0
    a.total_blocks = int(total_blocks)
    a.max_seq_blocks = int(max_seq_blocks)
    return a


def decode_plan(args: "_capi.DecodeArgs") -> dict:
    """Split-K plan the library picks for these arguments."""
    split, nsplit, tc = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
    ws = ctypes.c_size_t()
    _native.check(_native.lib().ouro_decode_plan(ctypes.byref(args), ctypes.byref(split),
                                                 ctypes.byref(nsplit), ctypes.byref(ws),
                                                 ctypes.byref(tc)), "decode plan")
    tc_used = bool(tc.value)
    # the library takes the stream-K form when asked for it, or on auto without a fixed split
    stream_k = tc_used and (args.kernel == 4 or (args.kernel == 0 and args.split_blocks == 0))
    return {"split_blocks": split.value, "max_splits": nsplit.value,
            "workspace_bytes": ws.value, "tensor_cores": tc_used, "stream_k": stream_k,
            "launches": 3 if stream_k else (2 if nsplit.value > 1 else 1)}


class DecodeCall:
    """A prepared decode launch: validated, device-resident arguments.

    Building one does the checks and conversions once; :meth:`launch` then
    only enqueues the kernels on the current stream (no host work besides the
    C call), so a serving loop or a CUDA graph can replay it.

    ``total_blocks`` (sum of ceil(keys / 64) over the batch) and
    ``max_seq_blocks`` (a bound on any sequence's blocks) are optional host
    figures for the split-K plan: with them the chunks are sized from the
    batch's real work and the workspace from its longest sequence instead of
    from the page-table width. Keys beyond ``max_seq_blocks * 64`` are not
    read and set status bit 1.

    ``out_ptr`` (instead of ``out``) is the raw device address of a contiguous
    [S, Hq, D] buffer in the cache dtype, for rows that live in memory torch does
    not own (another GPU's buffer mapped by CUDA IPC); :meth:`launch` then
    returns None.
    """

    def __init__(self, page_table, q, k_cache, v_cache, seq_lens, cos, sin, *, positions=None,
                 mask=None, scope=None, causal=False, softmax_scale=None, out=None,
                 validate=True, split_blocks=0, kernel="auto", workspace=None, status=None,
                 total_blocks=0, max_seq_blocks=0, out_ptr=None):
        _require_cuda()
        if kernel not in _KERNELS:
            raise RuntimeError(f"kernel must be one of {sorted(_KERNELS)}, got {kernel!r}")
        device = _device_of(k_cache, q, page_table, v_cache)
        k_cache = _on(k_cache, device)
        v_cache = _on(v_cache, device)
        if k_cache.dim() != 4:
            raise RuntimeError("k_cache must be [n_phys, Hkv, 64, D]")
        n_phys, Hkv, blk, D = k_cache.shape
        if blk != BLOCK_SIZE:
            raise RuntimeError(f"k_cache block dim must be {BLOCK_SIZE}, got {blk}")
        if v_cache.shape != k_cache.shape or v_cache.dtype != k_cache.dtype:
            raise RuntimeError("k/v caches must share the [n_phys, Hkv, 64, D] layout and dtype")
        if D < 2 or D % 2 != 0:
            raise RuntimeError(f"head dim must be even for half-split RoPE, got {D}")
        q = _on(q, device, k_cache.dtype)
        if q.dim() != 3 or q.shape[2] != D:
            raise RuntimeError(f"q must be [S, Hq, {D}], got {tuple(q.shape)}")
        S, Hq = q.shape[0], q.shape[1]
        if Hq % Hkv != 0:
            raise RuntimeError(f"query heads {Hq} must be a multiple of KV heads {Hkv}")
        page_table = _on(page_table, device)
        if page_table.dtype not in (torch.int32, torch.int64):
            raise RuntimeError(f"page_table must be int32/int64, got {page_table.dtype}")
        page_table = page_table.to(torch.int32)
        if page_table.dim() != 2 or page_table.shape[0] != S:
            raise RuntimeError(f"page_table must be [S={S}, max_blocks]")
        seq_lens = _on(seq_lens, device)
        if seq_lens.dtype not in (torch.int32, torch.int64):
            raise RuntimeError(f"seq_lens must be int32/int64, got {seq_lens.dtype}")
        seq_lens = seq_lens.to(torch.int32)
        if tuple(seq_lens.shape) != (S,):
            raise RuntimeError(f"seq_lens must have shape [{S}], got {tuple(seq_lens.shape)}")
        cos = _on(cos, device, torch.float32)
        sin = _on(sin, device, torch.float32)
        max_b = page_table.shape[1]
        if cos.dim() != 2 or cos.shape != sin.shape or cos.shape[1] != D // 2:
            raise RuntimeError(f"rope tables must be [max_positions, {D // 2}]")
        if cos.shape[0] < max_b * BLOCK_SIZE:
            raise RuntimeError(
                f"rope tables must cover {max_b * BLOCK_SIZE} positions, got {cos.shape[0]}")
        positions = _on(positions, device, torch.int32)
        if positions is not None and tuple(positions.shape) != (S,):
            raise RuntimeError(f"positions must have shape [{S}]")
        mask_arg = None
        if mask is not None:
            mask = _on(mask, device)
            validate_mask_shape(tuple(mask.shape), num_seqs=S, num_q_blocks=max_b,
                                num_kv_blocks=max_b)
            mask = mask.to(torch.int8).contiguous()
            mask_arg = (mask, _broadcast_strides(tuple(mask.shape), (S, max_b, max_b)))
        scope_arg = _scope_tensors(scope, S, device) if scope is not None else None
        if validate:
            validate_page_table(page_table, seq_lens, n_phys)
        if out_ptr is not None:
            if out is not None:
                raise RuntimeError("pass out or out_ptr, not both")
            if int(out_ptr) % 16 != 0:
                raise RuntimeError("out_ptr must be 16-byte aligned")
        elif out is None:
            out = torch.empty((S, Hq, D), dtype=k_cache.dtype, device=device)
        elif out.shape != (S, Hq, D) or out.dtype != k_cache.dtype or not out.is_contiguous():
            raise RuntimeError(f"out must be a contiguous [S, Hq, D] {k_cache.dtype} tensor")
        self._keep = (page_table, q, k_cache, v_cache, seq_lens, cos, sin, positions, mask_arg,
                      scope_arg)
        self.out = out
        self.device = device
        self.status = status
        if total_blocks < 0 or max_seq_blocks < 0:
            raise RuntimeError("total_blocks and max_seq_blocks must be >= 0 (0 = unknown)")
        args = _decode_args(page_table, q, k_cache, v_cache, seq_lens, cos, sin, positions,
                            mask_arg, scope_arg, causal, softmax_scale, split_blocks, kernel, out,
                            None, status, total_blocks, max_seq_blocks)
        if out_ptr is not None:
            args.out = int(out_ptr)
        self.plan = decode_plan(args)
        if self.plan["workspace_bytes"]:
            need = self.plan["workspace_bytes"]
            if workspace is None:
                workspace = torch.empty(-(-need // 16) * 4, dtype=torch.float32, device=device)
            elif workspace.numel() * workspace.element_size() < need:
                raise RuntimeError(f"workspace too small: need {need} bytes")
            args.workspace = _ptr(workspace)
            args.workspace_bytes = workspace.numel() * workspace.element_size()
        self.workspace = workspace
        self.args = args

    def launch(self):
        _native.check(_native.lib().ouro_paged_decode(ctypes.byref(self.args),
                                                      _stream_handle(self.device)), "decode")
        return self.out


def block_attention_decode(page_table, q, k_cache, v_cache, seq_lens, cos, sin, *,
                           positions=None, mask=None, scope=None, causal=False,
                           softmax_scale=None, out=None, validate=True, split_blocks=0,
                           kernel="auto", workspace=None, status=None, total_blocks=0,
                           max_seq_blocks=0):
    """Paged decode attention: one query token per sequence.

    Args:
        page_table: [S, max_blocks] int32/int64; row s lists the physical
            blocks of sequence s, PAD_ID (-1) past its chain
            (:func:`src.block_table.build_page_table` / ``export_page_table``).
        q: [S, Hq, D] query of the token being decoded (un-rotated).
        k_cache, v_cache: [n_phys, Hkv, 64, D] paged caches (fp32/fp16/bf16);
            query head h reads KV head h // (Hq / Hkv).
        seq_lens: [S] keys per sequence (the decoded token's K/V included).
        cos, sin: [max_positions, D/2] fp32 RoPE tables (half-split pairs).
        positions: optional [S] query positions (default seq_len - 1).
        mask: optional block mask broadcastable to [S, max_blocks, max_blocks];
            the query's row is positions // 64, zero entries drop whole blocks.
        scope: optional ``(tags [S, L], span [S, 2])`` token scope
            (:func:`src.scoping_mask.decode_scope`): key j is kept when
            tags[s, j] or span[s,0] <= j < span[s,1].
        causal: keep only keys j <= positions[s].
        softmax_scale: default 1/sqrt(D).
        validate: check the page table on the device first (one 8-byte read
            back; raises RuntimeError with the reference's messages).
        split_blocks / kernel / workspace / status / total_blocks /
            max_seq_blocks: launch controls and planning figures; see
            :class:`DecodeCall`.

    Returns:
        [S, Hq, D] tensor in the cache dtype.
    """
    call = DecodeCall(page_table, q, k_cache, v_cache, seq_lens, cos, sin, positions=positions,
                      mask=mask, scope=scope, causal=causal, softmax_scale=softmax_scale,
                      out=out, validate=validate, split_blocks=split_blocks, kernel=kernel,
                      workspace=workspace, status=status, total_blocks=total_blocks,
                      max_seq_blocks=max_seq_blocks)
    return call.launch()


# ---------------------------------------------------------------------------
# Multi-row attention: the reference's block_attention and chunked prefill
# ---------------------------------------------------------------------------


def _rows_args(q, q_paged, k_cache, v_cache, page_table, seq_lens, q_start, cos, sin, bias,
               mask, out, status, Hq, Lq, causal, softmax_scale, kernel):
    n_phys, Hkv, _, D = k_cache.shape
    a = _capi.AttentionArgs()
    a.q, a.q_paged = _ptr(q), 1 if q_paged else 0
    a.k_cache, a.v_cache = _ptr(k_cache), _ptr(v_cache)
    a.page_table, a.seq_lens, a.q_start = _ptr(page_table), _ptr(seq_lens), _ptr(q_start)
    a.cos, a.sin = _ptr(cos), _ptr(sin)
    if bias is not None:
        a.bias = _ptr(bias[0])
        a.bias_stride_s, a.bias_stride_h, a.bias_stride_q, a.bias_stride_k = bias[1]
    if mask is not None:
        a.block_mask = _ptr(mask[0])
        a.mask_stride_s, a.mask_stride_q, a.mask_stride_k = mask[1]
    a.out, a.status = _ptr(out), _ptr(status)
    a.num_seqs, a.num_q_heads, a.num_kv_heads, a.head_dim = page_table.shape[0], Hq, Hkv, D
    a.q_len = Lq
    a.max_blocks, a.num_phys_blocks, a.max_positions = page_table.shape[1], n_phys, cos.shape[0]
    a.dtype = _dtype_code(k_cache.dtype)
    a.causal = 1 if causal else 0
    a.kernel = _KERNELS[kernel]
    a.softmax_scale = float(softmax_scale) if softmax_scale is not None else 0.0
    return a


def _launch_rows(args, device):
    _native.check(_native.lib().ouro_paged_attention(ctypes.byref(args), _stream_handle(device)),
                  "paged attention")


def _as_int32(t, name: str):
    if t.dtype not in (torch.int32, torch.int64):
        raise RuntimeError(f"{name} must be int32/int64, got {t.dtype}")
    return t.to(torch.int32).contiguous()


def block_attention(page_table, q_cache, k_cache, v_cache, seq_lens, cos, sin, bias=None,
                    mask=None, softmax_scale: float | None = None, *, kernel: str = "auto"):
    """Full paged self-attention: the reference's ``block_attention``, on B200.

    Same arguments, checks, error texts and result as the reference
    (src/kernels/block_attention.py:368-527):

    * ``page_table`` [S, max_blocks]: physical block of logical block n of
      sequence s, PAD_ID past the chain;
    * ``q_cache, k_cache, v_cache`` [n_phys, H, 64, D] (fp32/fp16/bf16);
    * ``seq_lens`` [S]: self-attention, query extent = key extent;
    * ``cos, sin`` [max_positions, D/2] fp32, half-split RoPE at absolute
      positions;
    * ``bias`` broadcastable to [S, H, Q, K], added to the scaled scores;
    * ``mask`` block mask broadcastable to [S, QB, KB], zero = KV block dropped;
    * ``softmax_scale`` defaults to 1/sqrt(D).
    * ``kernel`` (keyword, not in the reference): "auto" runs fp16/bf16 caches with
      head_dim 128 and no bias on the tcgen05 tensor-core kernel (keys rotated once
      into a scratch the call allocates: S x H x max_blocks x 64 x D elements) and
      everything else on the CUDA cores; "tc" / "simt" force one.

    Returns [S, H, max_len, D] in the cache dtype; rows past seq_lens[s] are 0.
    """
    _require_cuda()
    named = (page_table, q_cache, k_cache, v_cache, seq_lens, cos, sin)
    device = _device_of(*named, bias, mask)
    page_table, q_cache, k_cache, v_cache, seq_lens = (
        _on(t, device) for t in (page_table, q_cache, k_cache, v_cache, seq_lens))
    cos, sin = _on(cos, device, torch.float32), _on(sin, device, torch.float32)
    S, max_b = page_table.shape
    n_phys, H, blk, D = q_cache.shape
    if blk != BLOCK_SIZE:
        raise RuntimeError(f"q_cache block dim must be {BLOCK_SIZE}, got {blk}")
    if k_cache.shape != q_cache.shape or v_cache.shape != q_cache.shape:
        raise RuntimeError("q/k/v caches must share the [n_phys, H, 64, D] layout")
    if D < 32 or D % 2 != 0:
        raise RuntimeError(f"head dim must be even and >= 32 for half-dot RoPE, got {D}")
    if tuple(seq_lens.shape) != (S,):
        raise RuntimeError(f"seq_lens must have shape [{S}], got {tuple(seq_lens.shape)}")
    pt = _as_int32(page_table, "page_table")
    lens = _as_int32(seq_lens, "seq_lens")
    max_len = _validate_page_table(pt, lens, n_phys, with_max_len=True)
    if max_len == 0:
        raise RuntimeError("all sequences are empty")
    if cos.shape[0] < max_b * BLOCK_SIZE or sin.shape[0] < max_b * BLOCK_SIZE:
        raise RuntimeError(
            f"rope tables must cover {max_b * BLOCK_SIZE} positions, got {cos.shape[0]}")
    qb_max = -(-max_len // BLOCK_SIZE)
    bias_arg = mask_arg = None
    if bias is not None:
        bias = _on(bias, device)
        validate_bias_shape(tuple(bias.shape), num_seqs=S, num_heads=H, q_len=max_len,
                            kv_len=max_len)
        bias = bias.to(torch.float32).contiguous()
        bias_arg = (bias, _broadcast_strides(tuple(bias.shape), (S, H, max_len, max_len)))
    if mask is not None:
        mask = _on(mask, device)
        validate_mask_shape(tuple(mask.shape), num_seqs=S, num_q_blocks=qb_max,
                            num_kv_blocks=qb_max)
        mask = mask.to(torch.int8).contiguous()
        mask_arg = (mask, _broadcast_strides(tuple(mask.shape), (S, qb_max, qb_max)))
    q_c = q_cache.to(k_cache.dtype).contiguous()
    out = torch.zeros((S, H, max_len, D), dtype=k_cache.dtype, device=device)
    if kernel not in _KERNELS or _KERNELS[kernel] > 2:
        raise RuntimeError(f"kernel must be 'auto', 'tc' or 'simt', got {kernel!r}")
    args = _rows_args(q_c, True, k_cache, v_cache, pt, lens, None, cos, sin, bias_arg, mask_arg,
                      out, None, H, max_len, False, softmax_scale, kernel)
    need, tc = ctypes.c_size_t(), ctypes.c_int32()
    _native.check(_native.lib().ouro_attention_plan(ctypes.byref(args), ctypes.byref(need),
                                                    ctypes.byref(tc)), "attention plan")
    workspace = None
    if tc.value and need.value:
        workspace = torch.empty(need.value, dtype=torch.uint8, device=device)
        args.workspace, args.workspace_bytes = _ptr(workspace), need.value
    _launch_rows(args, device)
    return out


class PrefillCall:
    """A prepared chunked-prefill launch (checked once, then :meth:`launch` only enqueues)."""

    def __init__(self, page_table, q, k_cache, v_cache, q_start, seq_lens, cos, sin, *,
                 causal: bool = True, softmax_scale=None, out=None, validate: bool = True,
                 kernel: str = "auto", status=None, workspace=None, krot_valid=None,
                 scope=None, launch_seq: int = 0):
        """``scope`` (optional) is the batch's token scope ``(tags, lo, hi)``, each
        [S, W] with W a multiple of 16 covering seq_lens (from
        :func:`src.scoping_mask.prefill_scope`): the query at position i keeps
        key j when tags[s, j] or lo[s, i] <= j < hi[s, i] (Table 1).

        ``workspace`` (optional uint8 device tensor) is the tensor-core path's
        rotated-key scratch; pass the same tensor to the calls of one chunked
        prefill together with ``krot_valid`` ([S] int32: keys [0, krot_valid[s])
        already rotated there by an earlier call with the same caches, page-table
        width and RoPE tables) and each key is rotated once instead of once per
        chunk.

        ``launch_seq``: the call's position in a chain of launches that share
        ``workspace`` and follow each other on one stream (chunk k of a chunked
        prefill: k); 0 (the default) starts a chain. A launch's CTAs may be
        scheduled while the previous kernel on the stream finishes, and wait for
        it before they touch memory."""
        _require_cuda()
        if kernel not in _KERNELS:
            raise RuntimeError(f"kernel must be one of {sorted(_KERNELS)}, got {kernel!r}")
        device = _device_of(k_cache, q, page_table)
        k_cache, v_cache = _on(k_cache, device), _on(v_cache, device)
        n_phys, Hkv, blk, D = k_cache.shape
        if blk != BLOCK_SIZE:
            raise RuntimeError(f"k_cache block dim must be {BLOCK_SIZE}, got {blk}")
        if v_cache.shape != k_cache.shape or v_cache.dtype != k_cache.dtype:
            raise RuntimeError("k/v caches must share the [n_phys, Hkv, 64, D] layout and dtype")
        q = _on(q, device, k_cache.dtype)
        if q.dim() != 4 or q.shape[3] != D:
            raise RuntimeError(f"q must be [S, Hq, L, {D}], got {tuple(q.shape)}")
        S, Hq, L = q.shape[0], q.shape[1], q.shape[2]
        if Hq % Hkv != 0:
            raise RuntimeError(f"query heads {Hq} must be a multiple of KV heads {Hkv}")
        pt = _as_int32(_on(page_table, device), "page_table")
        if pt.dim() != 2 or pt.shape[0] != S:
            raise RuntimeError(f"page_table must be [S={S}, max_blocks]")
        lens = _as_int32(_on(seq_lens, device), "seq_lens")
        starts = _as_int32(_on(q_start, device), "q_start")
        if tuple(lens.shape) != (S,) or tuple(starts.shape) != (S,):
            raise RuntimeError(f"seq_lens and q_start must have shape [{S}]")
        cos, sin = _on(cos, device, torch.float32), _on(sin, device, torch.float32)
        if cos.dim() != 2 or cos.shape != sin.shape or cos.shape[1] != D // 2:
            raise RuntimeError(f"rope tables must be [max_positions, {D // 2}]")
        if cos.shape[0] < pt.shape[1] * BLOCK_SIZE:
            raise RuntimeError(
                f"rope tables must cover {pt.shape[1] * BLOCK_SIZE} positions, got {cos.shape[0]}")
        if validate:
            validate_page_table(pt, lens, n_phys)
        if out is None:
            out = torch.zeros((S, Hq, L, D), dtype=k_cache.dtype, device=device)
        elif out.shape != (S, Hq, L, D) or out.dtype != k_cache.dtype or not out.is_contiguous():
            raise RuntimeError(f"out must be a contiguous [S, Hq, L, D] {k_cache.dtype} tensor")
        self.out = out
        self.device = device
        self.args = _rows_args(q, False, k_cache, v_cache, pt, lens, starts, cos, sin, None, None,
                               out, status, Hq, L, causal, softmax_scale, kernel)
        if launch_seq < 0:
            raise RuntimeError("launch_seq must be >= 0")
        self.args.launch_seq = int(launch_seq)
        scope_keep = None
        if scope is not None:
            tags, lo, hi = scope
            tags = _on(torch.as_tensor(tags), device, torch.uint8).contiguous()
            lo = _as_int32(_on(torch.as_tensor(lo), device), "scope lo")
            hi = _as_int32(_on(torch.as_tensor(hi), device), "scope hi")
            if tags.dim() != 2 or tags.shape[0] != S or tags.shape[1] % 16 != 0:
                raise RuntimeError(f"scope tags must be [S={S}, W] with W a multiple of 16")
            if lo.shape != tags.shape or hi.shape != tags.shape:
                raise RuntimeError("scope lo / hi must have the shape of the tags")
            if tags.shape[1] < int(lens.max().item()):
                raise RuntimeError("scope arrays must cover every sequence length")
            self.args.scope_tags, self.args.scope_stride = _ptr(tags), tags.shape[1]
            self.args.scope_lo, self.args.scope_hi = _ptr(lo), _ptr(hi)
            scope_keep = (tags, lo, hi)
        need, tc = ctypes.c_size_t(), ctypes.c_int32()
        _native.check(_native.lib().ouro_attention_plan(ctypes.byref(self.args),
                                                        ctypes.byref(need), ctypes.byref(tc)),
                      "attention plan")
        self.tensor_cores = bool(tc.value)
        self.workspace = None
        if need.value:  # rotated-key scratch of the tensor-core path
            if workspace is None:
                workspace = torch.empty(need.value, dtype=torch.uint8, device=device)
            elif (workspace.dtype != torch.uint8 or workspace.device != device
                  or workspace.numel() < need.value or not workspace.is_contiguous()):
                raise RuntimeError(f"workspace must be a contiguous uint8 tensor on {device} "
                                   f"of at least {need.value} bytes")
            self.workspace = workspace
            self.args.workspace = _ptr(workspace)
            self.args.workspace_bytes = need.value
        if krot_valid is not None:
            krot_valid = _as_int32(_on(krot_valid, device), "krot_valid")
            if tuple(krot_valid.shape) != (S,):
                raise RuntimeError(f"krot_valid must have shape [{S}]")
            self.args.krot_valid = _ptr(krot_valid)
        self._keep = (q, k_cache, v_cache, pt, lens, starts, cos, sin, status, krot_valid,
                      scope_keep)

    def launch(self):
        _launch_rows(self.args, self.device)
        return self.out


def chunked_prefill_attention(page_table, q, k_cache, v_cache, q_start, seq_lens, cos, sin, *,
                              causal: bool = True, softmax_scale=None, out=None,
                              validate: bool = True, kernel: str = "auto", status=None,
                              workspace=None, krot_valid=None, scope=None):
    """Chunked prefill: q [S, Hq, L, D] rows at positions q_start[s] + i.

    Keys are every paged token j < seq_lens[s] (the chunk's own K/V already
    written into the cache), j <= q_start[s] + i when ``causal``. Query head h
    reads KV head h // (Hq / Hkv). Rows whose position is >= seq_lens[s] stay
    zero. fp16/bf16 with head_dim 128 run on the tcgen05 tensor-core kernel;
    other shapes and fp32 on CUDA cores. Returns [S, Hq, L, D] in the cache dtype.
    ``workspace`` / ``krot_valid``: reuse of the rotated-key scratch across the
    chunks of one prefill; ``scope``: the token scope (see :class:`PrefillCall`).
    """
    return PrefillCall(page_table, q, k_cache, v_cache, q_start, seq_lens, cos, sin,
                       causal=causal, softmax_scale=softmax_scale, out=out, validate=validate,
                       kernel=kernel, status=status, workspace=workspace,
                       krot_valid=krot_valid, scope=scope).launch()


def paged_kv_append(k_new, v_new, page_table, start, counts, k_cache, v_cache, *, status=None):
    """Writes new tokens into the paged caches (the [EXPAND] data step).

    ``k_new``/``v_new`` [S, Hkv, L, D]; token t < counts[s] of sequence s goes to
    position start[s] + t of its chain (block page_table[s][pos // 64], slot
    pos % 64). The chains must already cover those positions.
    """
    _require_cuda()
    device = _device_of(k_cache)
    if k_new.shape != v_new.shape or k_new.dim() != 4:
        raise RuntimeError("k_new / v_new must both be [S, Hkv, L, D]")
    S, Hkv, L, D = k_new.shape
    if k_cache.shape[1] != Hkv or k_cache.shape[3] != D or k_cache.shape[2] != BLOCK_SIZE:
        raise RuntimeError("new K/V heads and head_dim must match the cache")
    k_new = _on(k_new, device, k_cache.dtype)
    v_new = _on(v_new, device, k_cache.dtype)
    pt = _as_int32(_on(page_table, device), "page_table")
    st = _as_int32(_on(start, device), "start")
    ct = _as_int32(_on(counts, device), "counts")
    _native.check(_native.lib().ouro_kv_append(
        _ptr(k_new), _ptr(v_new), _ptr(pt), _ptr(st), _ptr(ct), _ptr(k_cache), _ptr(v_cache),
        S, Hkv, L, D, k_cache.element_size(), pt.shape[1], k_cache.shape[0], _ptr(status),
        _stream_handle(device)), "kv append")


def __getattr__(name: str):
    """Names of the reference module that this one deliberately does not provide.

    ``dense_reference`` (block_attention.py:538-595 of the reference) is the
    reference's fp32 torch check of this kernel, an O(T^2) CPU-capable
    computation; this module holds only the GPU path, so the check stays with
    the code it checks. Callers keep importing it from the reference checkout
    (``src.kernels.block_attention.dense_reference``), or use this
    repository's numpy restatement ``oracle.attention_oracle.dense_attention``
    (test infrastructure).
    """
    if name == "dense_reference":
        raise AttributeError(
            "dense_reference is not part of the B200 module: it is the reference's fp32 "
            "check, not the attention path. Import it from the reference checkout "
            "(src.kernels.block_attention.dense_reference) or use "
            "oracle.attention_oracle.dense_attention from this repository's tests")
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
