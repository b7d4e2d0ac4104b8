"""i8l_w8a8_mm_noalloc: the GEMM entry point for callers that cannot allocate device
memory (a host that hands out memory only from its own fixed arena, a latency-critical
path that must not reach cudaMalloc, a caller with no allocator binding).  It takes its
split-K scratch from a fixed array inside the library instead of a caller workspace.

Checked through the C ABI against i8l_w8a8_mm (the entry point with a caller
workspace) on a decode shape whose default tile splits K, so the scratch is used, on
two calls in a row: the outputs must be bit-identical, the tolerance every GEMM test in
this suite uses.  This file is collected last on purpose.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from int8_linear import _native
from int8_linear.kernel import Config
from oracle import gemm as og
from tests.gpu_util import bits, ints, np_

pytestmark = pytest.mark.gpu


def _args(a, w, sa, sb, bias, out):
    return (a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0),
            sa.data_ptr(), 1, sb.data_ptr(), 1,
            bias.data_ptr() if bias is not None else None, _native.BF16,
            out.data_ptr(), _native.I32 if out.dtype == torch.int32 else _native.BF16, out.stride(0),
            a.shape[0], w.shape[0], a.shape[1])


# Stream-K tiles (split=2): their split tiles reduce through the scratch.
CASES = [(1, 2048, 4096, Config(16, 128, split=2)), (16, 6144, 2048, Config(16, 128, split=2)),
         (33, 2048, 12288, Config(64, 128, split=2))]


@pytest.mark.parametrize("m,k,n,cfg", CASES, ids=lambda v: getattr(v, "name", v))
def test_noalloc_matches_workspace_entry_point(m, k, n, cfg):
    lib = _native.load()
    a, w = ints((m, k), 70 + m), ints((n, k), 71)
    g = torch.Generator().manual_seed(72)
    sa = (torch.rand((m, 1), generator=g) * 1e-2 + 1e-3).cuda()
    sb = (torch.rand((n, 1), generator=g) * 1e-3 + 1e-4).cuda()
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16).cuda()
    tile = cfg.as_tile()
    need = lib.i8l_workspace_size(m, n, k, ctypes.byref(tile))
    assert need > 0, "this shape should split K and so use scratch"
    stream = torch.cuda.current_stream().cuda_stream

    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device="cuda")
    want = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    _native.check(lib.i8l_w8a8_mm(*_args(a, w, sa, sb, bias, want), ctypes.byref(tile),
                                  ws.data_ptr(), ws.numel(), stream))
    for _ in range(2):  # the shared scratch must come back clean for the next call
        got = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        _native.check(lib.i8l_w8a8_mm_noalloc(*_args(a, w, sa, sb, bias, got), ctypes.byref(tile),
                                              stream))
        torch.cuda.synchronize()
        assert np.array_equal(bits(got), bits(want))
    raw = torch.empty((m, n), dtype=torch.int32, device="cuda")
    _native.check(lib.i8l_w8a8_mm_noalloc(*_args(a, w, sa, sb, bias, raw), ctypes.byref(tile),
                                          stream))
    assert np.array_equal(np_(raw), og.exact(np_(a), np_(w)))
    assert _native.read_status() == 0


def test_noalloc_rejects_problems_whose_scratch_does_not_fit():
    lib = _native.load()
    m, k, n = 4096, 2048, 12312          # stream-K 128x256 tiles need ~19 MB of scratch
    a, w = ints((m, k), 1), ints((n, k), 2)
    one = torch.ones(1, device="cuda")
    out = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    tile = Config(128, 256, split=2).as_tile()
    need = lib.i8l_workspace_size(m, n, k, ctypes.byref(tile))
    assert need > 8 << 20
    rc = lib.i8l_w8a8_mm_noalloc(a.data_ptr(), k, w.data_ptr(), k, one.data_ptr(), 0,
                                 one.data_ptr(), 0, None, 0, out.data_ptr(), _native.BF16, n,
                                 m, n, k, ctypes.byref(tile), torch.cuda.current_stream().cuda_stream)
    assert rc == _native.EWORKSPACE
    assert b"scratch" in lib.i8l_last_error()
