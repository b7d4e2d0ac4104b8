"""The tensor-parallel exchange kernels' bounded waits, on one GPU.

A descriptor whose "peer" buffer is this GPU's own makes rank 0 wait for a flag that
no one ever sets: the wait must give up after the descriptor's time limit, leave the
peer-wait bit in the status word and return, with the CUDA context still usable.
"""

from __future__ import annotations

import ctypes
import time

import pytest
import torch

from int8_linear import _native

pytestmark = pytest.mark.gpu

PEER_WAIT_BIT = 1 << 6


def _lonely_comm(timeout_ns: int, slot_bytes=1 << 16, max_rows=64):
    lib = _native.load()
    own = ctypes.c_void_p()
    handle = (ctypes.c_uint8 * _native.PEER_HANDLE_BYTES)()
    _native.check(lib.i8l_peer_alloc(lib.i8l_peer_buffer_bytes(slot_bytes, 2), ctypes.byref(own), handle))
    epochs = torch.zeros(max_rows, dtype=torch.int32, device="cuda")
    d = _native.I8LPeerComm()
    d.bases[0] = d.bases[1] = own.value   # "rank 1" is this GPU's own buffer: nobody signals
    d.epochs = epochs.data_ptr()
    d.rank, d.world, d.slot_bytes, d.max_rows, d.timeout_ns = 0, 2, slot_bytes, max_rows, timeout_ns
    return d, own, epochs


def test_a_peer_that_never_signals_ends_the_wait_with_a_status_bit():
    lib = _native.load()
    _native.clear_status()
    d, own, epochs = _lonely_comm(timeout_ns=50_000_000)   # 50 ms
    x = torch.randn((3, 256), device="cuda").to(torch.bfloat16)
    q = torch.empty((3, 256), dtype=torch.int8, device="cuda")
    s = torch.empty((3, 1), dtype=torch.float32, device="cuda")
    t0 = time.perf_counter()
    _native.check(lib.i8l_tp_quant_rows(ctypes.byref(d), x.data_ptr(), 256, _native.BF16, q.data_ptr(), 256,
                                        s.data_ptr(), 3, 256, 1, torch.cuda.current_stream().cuda_stream))
    status = _native.read_status()
    elapsed = time.perf_counter() - t0
    assert status & PEER_WAIT_BIT, status
    assert elapsed < 10.0
    assert int(epochs[0].item()) == 1          # the call still completed its epoch
    _native.clear_status()
    assert _native.read_status() == 0
    # The context is still usable.
    y = torch.ones(4, device="cuda") * 2
    assert float(y.sum()) == 8.0
    _native.check(lib.i8l_peer_free(own))


def test_declines_what_the_exchange_buffer_cannot_hold():
    lib = _native.load()
    d, own, _ = _lonely_comm(timeout_ns=1_000_000, slot_bytes=1024, max_rows=8)
    acc = torch.zeros((16, 64), dtype=torch.int32, device="cuda")
    one = torch.ones(1, device="cuda")
    out = torch.empty((16, 64), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_native.NotSupported):
        _native.check(lib.i8l_tp_allreduce_dequant(ctypes.byref(d), acc.data_ptr(), 64, one.data_ptr(), 0,
                                                   one.data_ptr(), 0, None, 0, out.data_ptr(), _native.BF16,
                                                   64, 16, 64, torch.cuda.current_stream().cuda_stream))
    _native.check(lib.i8l_peer_free(own))
