"""CUDA-core GEMMs that quantise their own activation in a prologue (split-5 tiles).

Each fused call must give exactly the bits of the two launches it replaces: the
standalone quantiser (add_rmsnorm_quant, per_token_quant, silu_mul_quant) followed by
w8a8_mm on the same tile; the residual output of the norm too.  The C entry points are
called directly, so a silent fallback to the two steps cannot pass for a supported case.
The chain to the oracle is closed by tests/test_quant_gpu.py (quantisers against the
reference's arithmetic) and tests/test_gemm_gpu.py (GEMM against the exact product).
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from int8_linear import Config, _native, w8a8_mm, w8a8_mm_quant_act
from int8_linear import fused_quant as fq
from int8_linear.kernel import rmsnorm_w8a8_mm, silu_mul_w8a8_mm
from oracle import gemm as og
from oracle import quant as oq
from oracle.numerics import to_bits
from tests.gpu_util import bits, ints, np_, rand

pytestmark = pytest.mark.gpu

ACT = {torch.bfloat16: _native.BF16, torch.float16: _native.F16}
WDT = {torch.bfloat16: _native.BF16, torch.float16: _native.F16, torch.float32: _native.F32}


def tile(m: int) -> Config:
    return Config(next(t for t in (1, 2, 4, 8) if t >= m), 0, split=5)


def weight(n, k, seed):
    w = ints((n, k), seed)
    g = torch.Generator().manual_seed(seed)
    sb = (torch.rand((n, 1), generator=g) * 1e-3 + 1e-4).cuda()
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16).cuda()
    return w, sb, bias


def call_norm(x, res, gamma, w, sb, bias, cfg, out_dtype=torch.bfloat16):
    m, k = x.shape
    n = w.shape[0]
    out = torch.full((m, n), float("nan"), dtype=out_dtype, device="cuda")
    rout = torch.full_like(x, float("nan")) if res is not None else None
    rc = _native.load().i8l_rmsnorm_w8a8_mm(
        x.data_ptr(), x.stride(0), res.data_ptr() if res is not None else None,
        res.stride(0) if res is not None else 0, gamma.data_ptr(), ACT[x.dtype], WDT[gamma.dtype],
        1e-6, 1, rout.data_ptr() if rout is not None else None, rout.stride(0) if rout is not None else 0,
        w.data_ptr(), w.stride(0), sb.data_ptr(), 1, bias.data_ptr() if bias is not None else None,
        _native.BF16, out.data_ptr(), {torch.bfloat16: _native.BF16, torch.float16: _native.F16,
                                        torch.float32: _native.F32, torch.int32: _native.I32}[out_dtype],
        out.stride(0), m, n, k, ctypes.byref(cfg.as_tile()), torch.cuda.current_stream().cuda_stream)
    return rc, out, rout


@pytest.mark.parametrize("m", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("k,n", [(2048, 4096), (2048, 12288), (1024, 1000), (4096, 6144)])
@pytest.mark.parametrize("has_res", [False, True])
def test_norm_prologue_equals_the_two_launches(m, k, n, has_res):
    x, r = rand((m, k), 200 + m), rand((m, k), 201 + m) if has_res else None
    gamma = (1.0 + 0.1 * rand((k,), 202, dtype=torch.float32)).to(torch.bfloat16)
    w, sb, bias = weight(n, k, 203 + k)
    cfg = tile(m)
    rc, got, rout = call_norm(x, r, gamma, w, sb, bias, cfg)
    if k == 4096 and cfg.bm == 8:     # 8 tokens x 2 vectors per thread: more than the prologue holds
        assert rc == _native.ENOTSUP
        return
    assert rc == _native.OK, _native.load().i8l_last_error()
    q, s, r_want = fq.add_rmsnorm_quant(x, r, gamma, 1e-6)
    want = w8a8_mm(q, w.t(), s, sb, torch.bfloat16, bias, config=cfg)
    assert np.array_equal(bits(got), bits(want))
    if has_res:
        assert torch.equal(rout, r_want)
    # and the oracle on the same inputs: the quantiser within the reference tolerance,
    # the GEMM of that quantised activation bit-exact
    q0, s0, _ = oq.ref_norm(np_(x), np_(r) if has_res else None, np_(gamma), 1e-6,
                            quantiser=oq.quant_ieee, kernel_order=True)
    assert oq.compare_int8(np_(q), np_(s), q0, s0).ok()
    acc = og.exact(np_(q), np_(w))
    assert np.array_equal(bits(got), to_bits(og.epilogue_f32(acc, np_(s), np_(sb), np_(bias)), "bf16"))


@pytest.mark.parametrize("gdt", [torch.float16, torch.float32])
@pytest.mark.parametrize("adt", [torch.bfloat16, torch.float16])
def test_norm_prologue_dtypes(adt, gdt):
    m, k, n = 3, 2048, 2048
    x, r = rand((m, k), 210, dtype=adt), rand((m, k), 211, dtype=adt)
    gamma = (1.0 + 0.1 * rand((k,), 212, dtype=torch.float32)).to(gdt)
    w, sb, bias = weight(n, k, 213)
    rc, got, rout = call_norm(x, r, gamma, w, sb, bias, tile(m))
    assert rc == _native.OK, _native.load().i8l_last_error()
    q, s, r_want = fq.add_rmsnorm_quant(x, r, gamma, 1e-6)
    assert np.array_equal(bits(got), bits(w8a8_mm(q, w.t(), s, sb, torch.bfloat16, bias, config=tile(m))))
    assert torch.equal(rout, r_want)


@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("i,n", [(6144, 2048), (1024, 1000), (2048, 4096)])
@pytest.mark.parametrize("round_silu", [False, True])
@pytest.mark.parametrize("precise", [True, False])
def test_silu_prologue_equals_the_two_launches(m, i, n, round_silu, precise):
    gu = rand((m, 2 * i), 220 + m)
    w, sb, bias = weight(n, i, 221 + i)
    cfg = tile(m)
    out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    rc = _native.load().i8l_silu_mul_w8a8_mm(
        gu.data_ptr(), gu.stride(0), _native.BF16, int(precise), int(round_silu), w.data_ptr(), w.stride(0),
        sb.data_ptr(), 1, bias.data_ptr(), _native.BF16, out.data_ptr(), _native.BF16, out.stride(0),
        m, n, i, ctypes.byref(cfg.as_tile()), torch.cuda.current_stream().cuda_stream)
    assert rc == _native.OK, _native.load().i8l_last_error()
    q, s = fq.silu_mul_quant(gu, precise, round_silu)
    want = w8a8_mm(q, w.t(), s, sb, torch.bfloat16, bias, config=cfg)
    assert np.array_equal(bits(out), bits(want))
    # the Python entry gives the same (fused where it can, the two steps where not)
    assert np.array_equal(bits(silu_mul_w8a8_mm(gu, w.t(), sb, torch.bfloat16, bias, precise_div=precise,
                                                round_silu=round_silu, config=cfg)), bits(want))


@pytest.mark.parametrize("m", [1, 3, 8])
@pytest.mark.parametrize("k,n,ld", [(2048, 2048, 4096), (2048, 1000, 2048), (6144, 2048, 6144)])
def test_quant_prologue_equals_the_two_launches(m, k, n, ld):
    """o_proj's input: the per-token quantiser of a column slice (row stride ld)."""
    full = rand((m, ld), 230 + m)
    x = full[:, :k]
    w, sb, bias = weight(n, k, 231 + k)
    cfg = tile(m)
    got = w8a8_mm_quant_act(x, w.t(), sb, torch.bfloat16, bias, config=cfg)
    q, s = fq.per_token_quant(x)
    want = w8a8_mm(q, w.t(), s, sb, torch.bfloat16, bias, config=cfg)
    assert np.array_equal(bits(got), bits(want))
    q0, s0 = oq.quant_ieee(np_(x))
    assert np.array_equal(np_(q), q0) and np.array_equal(np_(s), s0)


def test_python_entry_falls_back_for_batches_the_prologue_does_not_hold():
    """8 tokens of K=4096: the fused kernel declines, rmsnorm_w8a8_mm runs the two steps."""
    m, k, n = 8, 4096, 1024
    x, r = rand((m, k), 240), rand((m, k), 241)
    gamma = torch.ones(k, dtype=torch.bfloat16, device="cuda")
    w, sb, _ = weight(n, k, 242)
    got, rout = rmsnorm_w8a8_mm(x, r, gamma, 1e-6, w.t(), sb, config=tile(m))
    q, s, r_want = fq.add_rmsnorm_quant(x, r, gamma, 1e-6)
    assert np.array_equal(bits(got), bits(w8a8_mm(q, w.t(), s, sb, config=tile(m))))
    assert torch.equal(rout, r_want)
    assert _native.read_status() == 0
