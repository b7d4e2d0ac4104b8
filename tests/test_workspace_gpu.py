"""The Python layer's split-K workspaces and CUDA graphs.

Stream-K tiles (split=2) reduce their split tiles through a zero-filled workspace that
every kernel leaves zeroed.  The workspace for captured calls is created, and zeroed,
outside any capture (int8_linear.kernel.workspace), so graphs captured one after another
share a clean buffer whichever of them is replayed first; a first call made inside a
capture is refused with a clear error; and reset_workspaces (run by clear_status and by
a non-zero read_status) zeroes stale partial sums.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from int8_linear import Config, _native, kernel, w8a8_mm
from oracle import gemm as og
from tests.gpu_util import ints, np_

pytestmark = pytest.mark.gpu

SK = Config(16, 128, split=2)   # stream-K decode tile: its split tiles use the workspace


def case(m, k, n, seed):
    a, w = ints((m, k), seed), ints((n, k), seed + 1)
    return a, w, og.exact(np_(a), np_(w))


def one():
    return torch.ones(1, device="cuda")


@pytest.fixture
def fresh_workspaces(monkeypatch):
    """Start from no cached workspaces (the module's state is restored afterwards)."""
    monkeypatch.setattr(kernel, "_workspaces", {})
    monkeypatch.setattr(kernel, "_capture_workspaces", {})
    yield


def test_two_graphs_replayed_in_either_order(fresh_workspaces):
    a1, w1, want1 = case(1, 2048, 4096, 10)
    a2, w2, want2 = case(16, 6144, 2048, 20)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):                      # warm-up outside any capture
        w8a8_mm(a1, w1.t(), one(), one(), raw=True, config=SK)
        w8a8_mm(a2, w2.t(), one(), one(), raw=True, config=SK)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g1, g2 = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g1):
        o1 = w8a8_mm(a1, w1.t(), one(), one(), raw=True, config=SK)
    with torch.cuda.graph(g2):
        o2 = w8a8_mm(a2, w2.t(), one(), one(), raw=True, config=SK)
    for _ in range(2):
        o2.zero_()
        g2.replay()                                    # the second graph first
        torch.cuda.synchronize()
        assert np.array_equal(np_(o2), want2)
        o1.zero_()
        g1.replay()
        torch.cuda.synchronize()
        assert np.array_equal(np_(o1), want1)
    # eager calls on the current stream are unaffected
    assert np.array_equal(np_(w8a8_mm(a1, w1.t(), one(), one(), raw=True, config=SK)), want1)
    assert _native.read_status() == 0


def test_first_call_inside_a_capture_is_refused(fresh_workspaces):
    a, w, _ = case(1, 2048, 4096, 30)
    g = torch.cuda.CUDAGraph()
    with pytest.raises(RuntimeError, match="warm-up"):
        with torch.cuda.graph(g):
            w8a8_mm(a, w.t(), one(), one(), raw=True, config=SK)
    torch.cuda.synchronize()
    # after a call outside the capture, capturing works
    w8a8_mm(a, w.t(), one(), one(), raw=True, config=SK)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = w8a8_mm(a, w.t(), one(), one(), raw=True, config=SK)
    g.replay()
    torch.cuda.synchronize()
    assert np.array_equal(np_(out), og.exact(np_(a), np_(w)))


def test_clear_status_rezeroes_stale_workspaces(fresh_workspaces):
    a, w, want = case(16, 6144, 2048, 40)
    assert np.array_equal(np_(w8a8_mm(a, w.t(), one(), one(), raw=True, config=SK)), want)
    # what a kernel that gave up a wait could leave behind: non-zero counters and sums
    for ws in kernel._workspaces.values():
        ws.fill_(3)
    _native.clear_status()
    for ws in kernel._workspaces.values():
        assert int(ws.count_nonzero()) == 0
    assert np.array_equal(np_(w8a8_mm(a, w.t(), one(), one(), raw=True, config=SK)), want)
