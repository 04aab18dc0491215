"""The peer-memory exchange kernels on one GPU: the protocol in loopback and its bounded waits.

The sharded decode step (src.dist.DecodeShards, exchange="peer") moves rows between
processes with four kernels (publish, fetch, signal, collect) and uint64 step flags.
Here one process plays both sides on one GPU, with the flags in a buffer from
ouro_ipc_alloc: publish permutes rows and raises a ready flag, fetch copies once the
flag has reached the step, signal raises a done flag, collect restores the order.
A flag that nothing raises makes fetch and collect give up after their time limit:
status bit 2 is set, nothing is copied and the call returns (no fault, no hang).
"""

import ctypes
import time

import pytest
import torch

from src import _native
from src.kernels import _capi  # noqa: F401  (registers the exchange symbols)

pytestmark = pytest.mark.gpu


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _flags(nbytes=4096):
    p = ctypes.c_void_p()
    _native.check(_native.lib().ouro_ipc_alloc(nbytes, ctypes.byref(p)), "ipc alloc")
    return p.value


def test_loopback_publish_fetch_signal_collect(cuda):
    lib = _native.lib()
    flags = _flags()
    rows, row_bytes = 37, 256
    q = torch.randn(rows, row_bytes // 4, device="cuda")
    perm = torch.randperm(rows, device="cuda")
    q_perm = torch.empty_like(q)
    ready = torch.tensor([flags], dtype=torch.int64, device="cuda")  # this GPU's own flag
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for step in (1, 2, 3):
        _native.check(lib.ouro_shard_publish(q.data_ptr(), perm.data_ptr(), q_perm.data_ptr(),
                                             rows, row_bytes, ready.data_ptr(), 1, step,
                                             _stream()), "publish")
        got = torch.zeros_like(q)
        _native.check(lib.ouro_shard_fetch(flags, step, 2_000_000_000, q_perm.data_ptr(),
                                           got.data_ptr(), rows * row_bytes, None, None, 0,
                                           status.data_ptr(), _stream()), "fetch")
        _native.check(lib.ouro_shard_signal(flags + 64, step, _stream()), "signal")
        back = torch.zeros_like(q)
        inv = torch.argsort(perm)
        _native.check(lib.ouro_shard_collect(flags + 64, 1, 8, step, 2_000_000_000,
                                             got.data_ptr(), inv.data_ptr(), back.data_ptr(),
                                             rows, row_bytes, status.data_ptr(), _stream()),
                      "collect")
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert torch.equal(got, q[perm]) and torch.equal(back, q)
    _native.check(lib.ouro_ipc_free(flags), "ipc free")


def test_fetch_and_collect_give_up_when_no_flag_rises(cuda):
    lib = _native.lib()
    flags = _flags()
    src = torch.arange(1024, dtype=torch.float32, device="cuda")
    dst = torch.zeros_like(src)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    t0 = time.time()
    # step 5 is never published: the fetch waits 20 ms, then reports and copies nothing
    _native.check(lib.ouro_shard_fetch(flags, 5, 20_000_000, src.data_ptr(), dst.data_ptr(),
                                       4096, None, None, 0, status.data_ptr(), _stream()),
                  "fetch")
    torch.cuda.synchronize()
    assert int(status.item()) & 2
    assert dst.abs().sum().item() == 0
    # one of two workers signals: the collect gives up as well, output untouched
    status.zero_()
    _native.check(lib.ouro_shard_signal(flags + 64, 5, _stream()), "signal")
    idx = torch.arange(8, dtype=torch.int64, device="cuda")
    out = torch.zeros(8, 32, device="cuda")
    _native.check(lib.ouro_shard_collect(flags + 64, 2, 8, 5, 20_000_000,
                                         src.data_ptr(), idx.data_ptr(), out.data_ptr(), 8, 128,
                                         status.data_ptr(), _stream()), "collect")
    torch.cuda.synchronize()
    assert int(status.item()) & 2 and out.abs().sum().item() == 0
    assert time.time() - t0 < 10
    # the context is still usable: the second worker's flag arrives and the collect runs
    status.zero_()
    _native.check(lib.ouro_shard_signal(flags + 128, 5, _stream()), "signal")
    _native.check(lib.ouro_shard_collect(flags + 64, 2, 8, 5, 2_000_000_000,
                                         src.data_ptr(), idx.data_ptr(), out.data_ptr(), 8, 128,
                                         status.data_ptr(), _stream()), "collect")
    torch.cuda.synchronize()
    assert int(status.item()) == 0 and torch.equal(out.reshape(-1), src[:256])
    _native.check(lib.ouro_ipc_free(flags), "ipc free")


def test_exchange_arguments_are_checked_on_the_host(cuda):
    lib = _native.lib()
    rc = lib.ouro_shard_fetch(None, 1, 1, None, None, 0, None, None, 0, None, _stream())
    assert rc == _native.OURO_EINVAL and "ready flag" in _native.last_error()
    rc = lib.ouro_shard_publish(None, None, None, 4, 100, None, 0, 1, _stream())
    assert rc == _native.OURO_EINVAL and "multiple of 16" in _native.last_error()
