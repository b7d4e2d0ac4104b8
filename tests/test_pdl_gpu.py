"""Programmatic dependent launch: kernels that start early must still see their
inputs.  Chains where each kernel consumes the previous one's output give
bit-identical results with PDL on and off, eagerly and inside CUDA graphs."""

from __future__ import annotations

import pytest
import torch

from int8_linear import _native, fused_quant as fq, set_pdl, w8a8_mm
from int8_linear.standin import StandinDecoder
from tests.gpu_util import ints, rand

pytestmark = pytest.mark.gpu


@pytest.fixture
def pdl_restore():
    before = _native.pdl_enabled()
    yield
    set_pdl(before)


def chain(x, ws, gamma):
    """norm -> GEMM -> quant -> GEMM -> SiLU -> GEMM, every step reading the last."""
    q, s, _ = fq.add_rmsnorm_quant(x, None, gamma, 1e-6)
    h = w8a8_mm(q, ws[0][0].t(), s, ws[0][1])
    q, s = fq.per_token_quant(h[:, :2048])
    gu = w8a8_mm(q, ws[1][0].t(), s, ws[1][1])
    q, s = fq.silu_mul_quant(gu)
    return w8a8_mm(q, ws[2][0].t(), s, ws[2][1])


@pytest.mark.parametrize("m", [1, 16, 100])
def test_dependent_chain_is_identical_with_pdl(m, pdl_restore):
    x = rand((m, 2048), 1)
    gamma = rand((2048,), 2, 0.1) + 1.0
    shapes = [(4096, 2048), (12288, 2048), (2048, 6144)]
    ws = [(ints((n, k), 3 + i), torch.rand((n, 1), device="cuda") * 1e-3 + 1e-4)
          for i, (n, k) in enumerate(shapes)]
    set_pdl(False)
    want = chain(x, ws, gamma)
    set_pdl(True)
    for _ in range(3):
        assert torch.equal(chain(x, ws, gamma), want)
    torch.cuda.synchronize()
    assert _native.read_status() == 0


@pytest.mark.parametrize("m", [1, 32])
def test_standin_graph_is_identical_with_pdl(m, pdl_restore):
    set_pdl(False)
    dec = StandinDecoder(m, layers=3)
    dec.capture().replay()
    torch.cuda.synchronize()
    want = dec.out.clone()
    set_pdl(True)
    dec2 = StandinDecoder(m, layers=3)
    g = dec2.capture()
    for _ in range(3):
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(dec2.out, want)
