"""ctypes mirrors of the attention argument structs in include/ouroboros_b200.h."""

from __future__ import annotations

import ctypes

from .. import _native

_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64


class DecodeArgs(ctypes.Structure):
    """``ouro_decode_args`` (field order and types must match the header)."""

    _fields_ = [
        ("q", _vp), ("k_cache", _vp), ("v_cache", _vp),
        ("page_table", _vp), ("seq_lens", _vp), ("positions", _vp),
        ("cos", _vp), ("sin", _vp),
        ("block_mask", _vp), ("mask_stride_s", _i64), ("mask_stride_q", _i64),
        ("mask_stride_k", _i64),
        ("scope_tags", _vp), ("scope_stride", _i64), ("scope_span", _vp),
        ("out", _vp), ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t), ("status", _vp),
        ("num_seqs", _i32), ("num_q_heads", _i32), ("num_kv_heads", _i32), ("head_dim", _i32),
        ("max_blocks", _i32), ("num_phys_blocks", _i32), ("max_positions", _i32),
        ("dtype", _i32), ("split_blocks", _i32), ("causal", _i32), ("kernel", _i32),
        ("softmax_scale", ctypes.c_float),
        ("total_blocks", _i64), ("max_seq_blocks", _i32),
    ]


_native.register("ouro_decode_plan", ctypes.c_int,
                 [ctypes.POINTER(DecodeArgs), ctypes.POINTER(_i32), ctypes.POINTER(_i32),
                  ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(_i32)])
_native.register("ouro_paged_decode", ctypes.c_int, [ctypes.POINTER(DecodeArgs), _vp])
_native.register("ouro_validate_page_table", ctypes.c_int,
                 [_vp, _vp, _i32, _i32, _i32, _vp, _vp])


class AttentionArgs(ctypes.Structure):
    """``ouro_attention_args`` (field order and types must match the header)."""

    _fields_ = [
        ("q", _vp), ("q_paged", _i32), ("k_cache", _vp), ("v_cache", _vp),
        ("page_table", _vp), ("seq_lens", _vp), ("q_start", _vp),
        ("cos", _vp), ("sin", _vp),
        ("bias", _vp), ("bias_stride_s", _i64), ("bias_stride_h", _i64),
        ("bias_stride_q", _i64), ("bias_stride_k", _i64),
        ("block_mask", _vp), ("mask_stride_s", _i64), ("mask_stride_q", _i64),
        ("mask_stride_k", _i64),
        ("out", _vp), ("status", _vp),
        ("num_seqs", _i32), ("num_q_heads", _i32), ("num_kv_heads", _i32), ("head_dim", _i32),
        ("q_len", _i32), ("max_blocks", _i32), ("num_phys_blocks", _i32),
        ("max_positions", _i32), ("dtype", _i32), ("causal", _i32), ("kernel", _i32),
        ("softmax_scale", ctypes.c_float),
        ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t), ("krot_valid", _vp),
        ("scope_tags", _vp), ("scope_stride", ctypes.c_int64), ("scope_lo", _vp),
        ("scope_hi", _vp), ("launch_seq", _i32),
    ]


_native.register("ouro_paged_attention", ctypes.c_int, [ctypes.POINTER(AttentionArgs), _vp])
_native.register("ouro_attention_plan", ctypes.c_int,
                 [ctypes.POINTER(AttentionArgs), ctypes.POINTER(ctypes.c_size_t),
                  ctypes.POINTER(_i32)])
_native.register("ouro_kv_append", ctypes.c_int,
                 [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
                  _vp, _vp])
_native.register("ouro_paged_decode_noalloc", ctypes.c_int, [ctypes.POINTER(DecodeArgs), _vp])

# Peer-memory exchange of the sharded decode step (src.dist.DecodeShards, exchange="peer").
_u64 = ctypes.c_uint64
_native.register("ouro_ipc_alloc", ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(_vp)])
_native.register("ouro_ipc_free", ctypes.c_int, [_vp])
_native.register("ouro_ipc_handle", ctypes.c_int, [_vp, _vp])
_native.register("ouro_ipc_open", ctypes.c_int, [_vp, ctypes.POINTER(_vp)])
_native.register("ouro_ipc_close", ctypes.c_int, [_vp])
_native.register("ouro_shard_publish", ctypes.c_int,
                 [_vp, _vp, _vp, _i64, _i64, _vp, _i32, _u64, _vp])
_native.register("ouro_shard_fetch", ctypes.c_int,
                 [_vp, _u64, _u64, _vp, _vp, _i64, _vp, _vp, _i64, _vp, _vp])
_native.register("ouro_shard_signal", ctypes.c_int, [_vp, _u64, _vp])
_native.register("ouro_shard_collect", ctypes.c_int,
                 [_vp, _i32, _i32, _u64, _u64, _vp, _vp, _vp, _i64, _i64, _vp, _vp])
