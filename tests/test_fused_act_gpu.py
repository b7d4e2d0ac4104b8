"""The GEMM with the activation's per-token quantisation fused into its loads
(w8a8_mm_quant_act, C entry i8l_w8a8_mm_quant_act): the same bits as the plain
per-token quantiser followed by w8a8_mm, and the int32 product equal to the oracle's
exact product of that quantisation."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from int8_linear import Config, NotSupported, _native, w8a8_mm, w8a8_mm_quant_act
from int8_linear import fused_quant as fq
from int8_linear.kernel import TOKEN_TILES, fused_act_config
from oracle import gemm as og
from tests.gpu_util import bits, ints, np_, rand

pytestmark = pytest.mark.gpu


def tok_tile(m):
    return next(t for t in TOKEN_TILES if t >= m)


def two_step(x, w, sb, out_dtype, bias, cfg, precise=True, raw=False):
    q, s = fq.per_token_quant(x, precise)
    return w8a8_mm(q, w.t(), s, sb, out_dtype, bias, config=cfg, raw=raw), q


def fused_direct(x, w, sb, out_dtype, bias, cfg, precise=True, raw=False):
    """Through the fused kernel only (no fall-back): the C entry must accept the tile."""
    lib = _native.load()
    m, k = x.shape
    n = w.shape[0]
    out = torch.empty((m, n), dtype=torch.int32 if raw else out_dtype, device="cuda")
    ws = torch.zeros(64 << 20, dtype=torch.uint8, device="cuda")
    code = {torch.bfloat16: _native.BF16, torch.float16: _native.F16, torch.float32: _native.F32}
    _native.check(lib.i8l_w8a8_mm_quant_act(
        x.data_ptr(), code[x.dtype], x.stride(0), int(precise), w.data_ptr(), w.stride(0),
        sb.data_ptr(), int(sb.numel() > 1), bias.data_ptr() if bias is not None else None,
        code[bias.dtype] if bias is not None else 0, out.data_ptr(),
        _native.I32 if raw else code[out_dtype], out.stride(0), m, n, k,
        cfg.as_tile(), ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream))
    return out


# (M, K, N, cluster, stages): direct loads need each CTA's k-blocks (K/128/cluster) in
# its ring of `stages` (0: the library's count, 5 for 16-token tiles, 3 for 64).
CASES = [(1, 2048, 2048, 4, 0), (2, 2048, 4096, 8, 0), (5, 6144, 2048, 8, 8), (16, 2048, 2048, 4, 0),
         (16, 1040, 1000, 2, 0), (40, 2048, 2048, 3, 6), (64, 2048, 2048, 3, 6), (3, 256, 520, 1, 0)]


@pytest.mark.parametrize("m,k,n,cluster,stages", CASES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fused_quant_matches_the_two_step_path(m, k, n, cluster, stages, dtype):
    x = rand((m, k), 300 + m, dtype=dtype)
    w = ints((n, k), 301)
    g = torch.Generator().manual_seed(302)
    sb = (torch.rand((n, 1), generator=g) * 1e-3 + 1e-4).cuda()
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16).cuda()
    split = 3 if cluster > 1 else 1
    cfg = Config(tok_tile(m), 128, split=split, cluster=cluster if split == 3 else 0, act=2,
                 ctas=0 if split == 3 else -(-n // 128), stages=stages)
    want_raw, q = two_step(x, w, sb, torch.bfloat16, None, cfg, raw=True)
    got_raw = fused_direct(x, w, sb, torch.bfloat16, None, cfg, raw=True)
    assert np.array_equal(np_(got_raw), np_(want_raw))
    assert np.array_equal(np_(got_raw), og.exact(np_(q).astype(np.int8), np_(w).astype(np.int8)))
    for out_dtype in (torch.bfloat16, torch.float32):
        want, _ = two_step(x, w, sb, out_dtype, bias, cfg)
        got = fused_direct(x, w, sb, out_dtype, bias, cfg)
        assert np.array_equal(bits(got), bits(want)), out_dtype


def test_column_slice_zero_rows_and_fast_division():
    """o_proj's input as the stand-in has it (the first 2048 columns of the qkv output,
    rows 4096 apart), with an all-zero row (scale 0) and a row with one large value."""
    m, k, n = 7, 2048, 2048
    qkv = rand((m, 4096), 310)
    qkv[2].zero_()
    qkv[4, 17] = 300.0
    x = qkv[:, :k]
    w = ints((n, k), 311)
    sb = (torch.rand((n, 1), generator=torch.Generator().manual_seed(312)) * 1e-3).cuda()
    cfg = Config(16, 128, split=3, cluster=4, act=2)
    for precise in (True, False):
        want, _ = two_step(x, w, sb, torch.bfloat16, None, cfg, precise=precise)
        got = fused_direct(x, w, sb, torch.bfloat16, None, cfg, precise=precise)
        assert np.array_equal(bits(got), bits(want)), precise
    assert not torch.any(got[2].float() != 0)


@pytest.mark.parametrize("m", [1, 2, 16, 64, 100, 300])
def test_public_api_fuses_where_it_can_and_falls_back_elsewhere(m):
    """The library's tiling (narrow or prefill tiles fall back to two launches): same bits."""
    k, n = 2048, 4096
    x = rand((m, k), 320 + m)
    w = ints((n, k), 321)
    sb = (torch.rand((n, 1), generator=torch.Generator().manual_seed(322)) * 1e-3).cuda()
    q, s = fq.per_token_quant(x)
    want = w8a8_mm(q, w.t(), s, sb, torch.bfloat16)
    got = w8a8_mm_quant_act(x, w.t(), sb, torch.bfloat16)
    assert np.array_equal(bits(got), bits(want))
    # an explicit swap_ab tiling whose k-blocks fit the ring goes through the fused kernel
    if m <= 16:
        cfg = fused_act_config(Config(16, 128, split=3, cluster=4))
        got = w8a8_mm_quant_act(x, w.t(), sb, torch.bfloat16, config=cfg)
        assert np.array_equal(bits(got), bits(want))
    assert _native.read_status() == 0


def test_declines_tiles_without_direct_loads():
    x = rand((16, 2048), 330)
    w = ints((2048, 2048), 331)
    sb = torch.ones(1, device="cuda")
    with pytest.raises(NotSupported, match="direct activation loads"):
        # cluster 2: 8 k-blocks per CTA, more than the ring's 5 stages
        fused_direct(x, w, sb, torch.bfloat16, None, Config(16, 128, split=3, cluster=2))


@pytest.mark.parametrize("m", [1, 5, 16, 40])
def test_standin_with_fused_o_proj_gives_the_same_step(m):
    """The stand-in decode step with o_proj's input quantised inside its GEMM equals the
    step with the separate quantiser, bit for bit, captured in a CUDA graph as well."""
    from int8_linear.standin import StandinDecoder

    dec = StandinDecoder(m, layers=3)
    want = dec.step().clone()
    dec.fuse_o_proj = True
    assert torch.equal(dec.step(), want)
    dec.capture().replay()
    torch.cuda.synchronize()
    assert torch.equal(dec.out, want)
