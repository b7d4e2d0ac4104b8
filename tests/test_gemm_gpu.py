"""The sm_100a W8A8 GEMM against the CPU oracle (oracle/gemm.py).

Mirrors the reference's tests/test_kernel.py: exact int32 products at its shapes,
other tilings, the 16 scaled-output cases, declines, CUDA-graph replay and odd
pointers; plus B200-specific coverage (every tile family, stream-K splits, ragged
M/N/K, bit-exact bf16/fp16 epilogue against the fp32 restatement).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from int8_linear import Config, NotSupported, _native, w8a8_mm
from int8_linear.kernel import TOKEN_TILES, choose_config
from oracle import gemm as og
from oracle.numerics import to_bits
from tests.gpu_util import bits, ints, np_, offset_ints

pytestmark = pytest.mark.gpu

SHAPES = [(1, 2048, 2048), (3, 2048, 1024), (17, 2048, 6144), (64, 2048, 2048), (100, 6144, 2048)]


def exact(a: torch.Tensor, w: torch.Tensor) -> np.ndarray:
    return og.exact(np_(a), np_(w))


def tok_tile(m):
    """The smallest swap_ab token tile that holds M rows."""
    return next(t for t in TOKEN_TILES if t >= m)


def one():
    return torch.ones(1, device="cuda")


@pytest.mark.parametrize("m,k,n", SHAPES)
def test_int32_product_is_exact(m, k, n):
    a, w = ints((m, k), 1), ints((n, k), 2)
    got = w8a8_mm(a, w.t(), one(), one(), raw=True)
    assert got.dtype == torch.int32 and np.array_equal(np_(got), exact(a, w))


TILINGS = [Config(t, 128) for t in (16, 32, 64, 128, 256)] + [
    Config(t, 128, split=2) for t in (16, 32, 64, 128, 256)] + [
    Config(128, 128, swap_ab=True), Config(128, 128), Config(128, 256),
    Config(16, 128, split=1), Config(128, 256, split=1), Config(128, 256, split=2),
    Config(64, 128, stages=2), Config(128, 256, stages=2, group_m=1),
    Config(32, 128, ctas=7, split=2), Config(128, 128, ctas=3, split=2),
    Config(16, 128, split=3), Config(32, 128, split=3, cluster=2), Config(64, 128, split=3, cluster=2),
    Config(16, 128, split=3, cluster=3), Config(16, 128, split=3, cluster=8),
    Config(16, 128, split=3, cluster=1), Config(64, 128, split=1, ctas=1000),
    Config(16, 128, split=3, cluster=2, store=2), Config(16, 128, split=3, cluster=3, store=2),
    Config(32, 128, split=3, cluster=2, store=2), Config(16, 128, split=3, cluster=4, store=1),
    Config(16, 128, split=2, store=2), Config(256, 128, store=2), Config(128, 256, store=2),
]


@pytest.mark.parametrize("config", TILINGS, ids=lambda c: c.name)
def test_exact_under_other_tilings(config):
    m, k, n = 256, 2048, 1024
    a, w = ints((m, k), 3), ints((n, k), 4)   # 256 tokens: several token tiles when bm < 256
    got = w8a8_mm(a, w.t(), one(), one(), raw=True, config=config)
    assert np.array_equal(np_(got), exact(a, w))


@pytest.mark.parametrize("m,k,n", [(1, 16, 1), (5, 48, 77), (130, 1040, 300), (300, 4096, 1000),
                                   (1000, 2048, 129), (777, 6144, 4096), (2048, 1024, 2048),
                                   (5, 2048, 1040), (300, 2048, 1040), (40, 512, 1048)])
def test_ragged_shapes_are_exact(m, k, n):
    """Sizes that are no multiple of any tile: TMA fills zeros past the edges and the
    epilogue masks the stores."""
    a, w = ints((m, k), m + k), ints((n, k), n)
    got = w8a8_mm(a, w.t(), one(), one(), raw=True)
    assert np.array_equal(np_(got), exact(a, w))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("per_row", [True, False])
@pytest.mark.parametrize("per_col", [True, False])
@pytest.mark.parametrize("use_bias", [True, False])
def test_scaled_output_matches_oracle(dtype, per_row, per_col, use_bias):
    m, k, n = 37, 2048, 1024
    a, w = ints((m, k), 5), ints((n, k), 6)
    g = torch.Generator().manual_seed(7)
    sa = (torch.rand((m, 1) if per_row else (1,), generator=g) * 1e-2 + 1e-3).cuda()
    sb = (torch.rand((n, 1) if per_col else (1,), generator=g) * 1e-2 + 1e-3).cuda()
    bias = torch.randn(n, generator=g).to(dtype).cuda() if use_bias else None
    got = w8a8_mm(a, w.t(), sa, sb, dtype, bias)
    assert got.dtype == dtype
    acc = exact(a, w)
    b = np_(bias) if use_bias else None
    # bit-exact against the fp32 restatement of the reference epilogue
    want = to_bits(og.epilogue_f32(acc, np_(sa), np_(sb), b),
                   {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}[dtype])
    assert np.array_equal(bits(got), want)
    # and within the reference's own 1% rule of the float64 layer
    term, ref = og.scaled_ref(acc, np_(sa), np_(sb), b)
    assert og.rel_error(np_(got), term, ref) < 1e-2


@pytest.mark.parametrize("m", [1, 16, 17, 64, 256, 300, 1024])
@pytest.mark.parametrize("k,n", [(2048, 4096), (6144, 2048)])
def test_decode_and_prefill_bf16_bit_exact(m, k, n):
    """Every default tile family and split path at Qwen3 widths, bf16 out with bias."""
    a, w = ints((m, k), 11 + m), ints((n, k), 12)
    g = torch.Generator().manual_seed(13)
    sa = (torch.rand((m, 1), generator=g) * 1e-2 + 1e-3).cuda()
    sb = (torch.rand((n, 1), generator=g) * 1e-3 + 1e-4).cuda()
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16).cuda()
    got = w8a8_mm(a, w.t(), sa, sb, torch.bfloat16, bias)
    want = to_bits(og.epilogue_f32(exact(a, w), np_(sa), np_(sb), np_(bias)), "bf16")
    assert np.array_equal(bits(got), want)


# (m, k, n, split, cluster): every token in one tile and each CTA's k-blocks in the ring.
DIRECT_ACT = [(1, 2048, 4096, 3, 4), (1, 2048, 2048, 3, 8), (5, 1040, 1000, 3, 4),
              (16, 2048, 4096, 3, 4), (17, 2048, 4096, 3, 4), (40, 256, 2048, 3, 2),
              (64, 384, 4096, 3, 2), (1, 4096, 1024, 3, 8), (1, 512, 4096, 1, 0),
              (3, 16, 300, 1, 0), (9, 272, 77, 3, 2)]


@pytest.mark.parametrize("m,k,n,split,cluster", DIRECT_ACT)
def test_direct_activation_loads_bit_exact(m, k, n, split, cluster):
    """Activation k-blocks copied into shared memory by the epilogue warps (plain loads,
    128-byte swizzle written by hand) give the same bits as the TMA path."""
    a, w = ints((m, k), 90 + m), ints((n, k), 91)
    g = torch.Generator().manual_seed(92)
    sa = (torch.rand((m, 1), generator=g) * 1e-2 + 1e-3).cuda()
    sb = (torch.rand((n, 1), generator=g) * 1e-3 + 1e-4).cuda()
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16).cuda()
    bm = tok_tile(m)
    want_raw = exact(a, w)
    want = to_bits(og.epilogue_f32(want_raw, np_(sa), np_(sb), np_(bias)), "bf16")
    for act in (1, 2):
        cfg = Config(bm, 128, swap_ab=True, split=split, cluster=cluster, act=act)
        assert np.array_equal(np_(w8a8_mm(a, w.t(), one(), one(), raw=True, config=cfg)), want_raw), act
        got = w8a8_mm(a, w.t(), sa, sb, torch.bfloat16, bias, config=cfg)
        assert np.array_equal(bits(got), want), act


def test_declines_direct_activation_loads_it_cannot_take():
    a, w = ints((17, 2048), 1), ints((1024, 2048), 2)
    with pytest.raises(NotSupported, match="direct activation"):   # two token tiles
        w8a8_mm(a, w.t(), one(), one(), config=Config(16, 128, split=3, cluster=4, act=2))
    with pytest.raises(NotSupported, match="direct activation"):   # 16 k-blocks per CTA
        w8a8_mm(a[:1], w.t(), one(), one(), config=Config(16, 128, split=1, act=2))


@pytest.mark.parametrize("m,k,n", [(256, 256, 256), (300, 1040, 1000), (1024, 2048, 4096), (4096, 2048, 12288),
                                   (513, 6144, 2056), (2000, 4096, 520)])
def test_cta_pair_tiles_bit_exact(m, k, n):
    """Two SMs per 256 x 256 tile (cta_group::2): each CTA loads its 128 token rows and
    half of the weight tile, the even CTA issues the 256-row MMAs; the int32 product
    and the bf16 output equal the one-CTA tiles'."""
    a, w = ints((m, k), 70 + m), ints((n, k), 71)
    g = torch.Generator().manual_seed(72)
    sa = (torch.rand((m, 1), generator=g) * 1e-2 + 1e-3).cuda()
    sb = (torch.rand((n, 1), generator=g) * 1e-3 + 1e-4).cuda()
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16).cuda()
    cfg = Config(128, 256, split=4)
    want = exact(a, w)
    assert np.array_equal(np_(w8a8_mm(a, w.t(), one(), one(), raw=True, config=cfg)), want)
    got = w8a8_mm(a, w.t(), sa, sb, torch.bfloat16, bias, config=cfg)
    assert np.array_equal(bits(got), to_bits(og.epilogue_f32(want, np_(sa), np_(sb), np_(bias)), "bf16"))
    for ctas in (2, 6):   # fewer pairs than tiles: each pair walks several tiles
        got = w8a8_mm(a, w.t(), one(), one(), raw=True, config=Config(128, 256, split=4, ctas=ctas))
        assert np.array_equal(np_(got), want), ctas


@pytest.mark.parametrize("m", [1, 2, 5, 16])
@pytest.mark.parametrize("k,n,cluster", [(2048, 4096, 8), (2048, 2048, 4), (6144, 2048, 8), (2048, 12288, 3),
                                         (1040, 1000, 4), (256, 520, 1), (2048, 4096, 2)])
def test_narrow_tiles_bit_exact(m, k, n, cluster):
    """Decode batches with the weight on the MMA's N side (64-row token tile x 256 weight
    rows, cluster split-K over DSMEM): same bits as the swap_ab tiles and the oracle."""
    a, w = ints((m, k), 60 + m), ints((n, k), 61)
    g = torch.Generator().manual_seed(62)
    sa = (torch.rand((m, 1), generator=g) * 1e-2 + 1e-3).cuda()
    sb = (torch.rand((n, 1), generator=g) * 1e-3 + 1e-4).cuda()
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16).cuda()
    cfg = Config(128, 256, split=3, cluster=cluster)
    want = exact(a, w)
    try:
        got = w8a8_mm(a, w.t(), one(), one(), raw=True, config=cfg)
    except NotSupported as e:   # partial sums larger than the ring for this batch
        assert "cluster size" in str(e) and m > 2, e
        return
    assert np.array_equal(np_(got), want)
    for dt, code in ((torch.bfloat16, "bf16"), (torch.float32, "f32")):
        got = w8a8_mm(a, w.t(), sa, sb, dt, bias, config=cfg)
        assert np.array_equal(bits(got), to_bits(og.epilogue_f32(want, np_(sa), np_(sb), np_(bias)), code)), dt


def test_split3_without_swap_above_16_tokens_is_a_128_token_cluster_tile():
    """Split 3 without swap_ab: narrow tiles up to 16 tokens, 128-token tiles with the
    weight on the MMA's N side and cluster split-K above."""
    a, w = ints((17, 2048), 1), ints((1024, 2048), 2)
    got = w8a8_mm(a, w.t(), one(), one(), raw=True, config=Config(128, 256, split=3, cluster=4))
    assert np.array_equal(np_(got), exact(a, w))


@pytest.mark.parametrize("m", [17, 64, 128, 200, 300])
@pytest.mark.parametrize("k,n", [(2048, 4096), (6144, 2048), (1040, 1000)])
@pytest.mark.parametrize("bn,cluster", [(256, 2), (256, 4), (128, 3), (128, 8)])
def test_cluster_split_on_128_token_tiles(m, k, n, bn, cluster):
    """Cluster split-K with the tokens on the 128-row MMA side and 128 or 256 weight rows
    per MMA: each CTA finishes its 16-column chunks (plain stores, 16-byte vectors where
    the row allows); ragged M, N and K; bf16 with bias and fp32."""
    a, w = ints((m, k), 400 + m), ints((n, k), 401)
    g = torch.Generator().manual_seed(402)
    sa = (torch.rand((m, 1), generator=g) * 1e-2 + 1e-3).cuda()
    sb = (torch.rand((n, 1), generator=g) * 1e-3 + 1e-4).cuda()
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16).cuda()
    cfg = Config(128, bn, split=3, cluster=cluster)
    want = exact(a, w)
    if cluster > (k + 127) // 128:
        with pytest.raises(NotSupported):
            w8a8_mm(a, w.t(), one(), one(), raw=True, config=cfg)
        return
    assert np.array_equal(np_(w8a8_mm(a, w.t(), one(), one(), raw=True, config=cfg)), want)
    got = w8a8_mm(a, w.t(), sa, sb, torch.bfloat16, bias, config=cfg)
    assert np.array_equal(bits(got), to_bits(og.epilogue_f32(want, np_(sa), np_(sb), np_(bias)), "bf16"))
    got32 = w8a8_mm(a, w.t(), sa, sb, torch.float32, config=cfg)
    assert np.array_equal(np_(got32), og.epilogue_f32(want, np_(sa), np_(sb), None))


def test_declines_a_cluster_whose_partial_sums_do_not_fit():
    # 16-token tiles: the one 16-column chunk goes to rank 0, 7 x 8 KB into a 2 x 18 KB ring
    a, w = ints((16, 2048), 1), ints((1024, 2048), 2)
    with pytest.raises(NotSupported, match="ring"):
        w8a8_mm(a, w.t(), one(), one(), config=Config(16, 128, split=3, cluster=8, stages=2))


def test_declines_shapes_the_kernel_does_not_take():
    a, w = ints((4, 100), 8), ints((64, 100), 9)
    with pytest.raises(NotSupported):
        w8a8_mm(a, w.t(), one(), one())
    with pytest.raises(NotSupported):       # N-contiguous [K, N] weight
        w8a8_mm(ints((4, 128), 1), ints((128, 64), 2), one(), one())
    with pytest.raises(NotSupported):
        w8a8_mm(ints((4, 128), 1), ints((64, 128), 2).t(), one().double(), one())
    with pytest.raises(ValueError):
        w8a8_mm(ints((4, 128), 1), ints((64, 128), 2).t(), torch.ones(3, device="cuda"), one())


def test_replays_inside_a_cuda_graph():
    m, k, n = 16, 2048, 2048
    a, w = ints((m, k), 10), ints((n, k), 11)
    sa = torch.full((m, 1), 1e-2, device="cuda")
    sb = torch.full((n, 1), 1e-2, device="cuda")
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        w8a8_mm(a, w.t(), sa, sb)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        static_out = w8a8_mm(a, w.t(), sa, sb)
    a.copy_(ints((m, k), 12))  # new input in the same buffer
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(static_out, w8a8_mm(a, w.t(), sa, sb))
    want = to_bits(og.epilogue_f32(exact(a, w), np_(sa), np_(sb)), "bf16")
    assert np.array_equal(bits(static_out), want)


def test_exact_on_an_odd_pointer_repeatedly():
    m, k, n = 5, 2048, 1024
    a, w = offset_ints((m, k), 23), ints((n, k), 24)
    for _ in range(3):
        assert np.array_equal(np_(w8a8_mm(a, w.t(), one(), one(), raw=True)), exact(a, w))


@pytest.mark.parametrize("split", [0, 2, 3])
def test_repeated_split_calls_leave_the_workspace_clean(split):
    """Split tiles reduce through the workspace (stream-K) or distributed shared memory
    (cluster) and leave nothing behind; many calls with different shapes in a row must
    each stay exact."""
    for i, (m, k, n) in enumerate([(1, 2048, 2048), (3, 6144, 2048), (16, 2048, 12288),
                                   (1, 14336, 4096), (40, 2048, 2048), (1, 2048, 2048)] * 2):
        a, w = ints((m, k), 30 + i), ints((n, k), 40 + i)
        cfg = Config(tok_tile(m), 128, split=split)
        assert np.array_equal(np_(w8a8_mm(a, w.t(), one(), one(), raw=True, config=cfg)), exact(a, w))
    assert _native.read_status() == 0


@pytest.mark.parametrize("store", [0, 1, 2])
@pytest.mark.parametrize("m", [1, 5, 16, 40, 64])
@pytest.mark.parametrize("k,n", [(2048, 4096), (2048, 2048), (6144, 2048), (2048, 12288), (14336, 4096)])
def test_cluster_split_bf16_bit_exact(m, k, n, store):
    """Decode shapes through cluster split-K, bf16 out with bias."""
    a, w = ints((m, k), 80 + m), ints((n, k), 81)
    g = torch.Generator().manual_seed(82)
    sa = (torch.rand((m, 1), generator=g) * 1e-2 + 1e-3).cuda()
    sb = (torch.rand((n, 1), generator=g) * 1e-3 + 1e-4).cuda()
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16).cuda()
    got = w8a8_mm(a, w.t(), sa, sb, torch.bfloat16, bias, config=Config(tok_tile(m), 128, split=3, store=store))
    want = to_bits(og.epilogue_f32(exact(a, w), np_(sa), np_(sb), np_(bias)), "bf16")
    assert np.array_equal(bits(got), want)


@pytest.mark.parametrize("m,n", [(1, 1040), (37, 1000), (300, 1040), (513, 2056), (200, 136)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_edge_tiles_bit_exact(m, n, dtype):
    """Output tiles that hang over M and N (some warps' store boxes lie wholly outside)."""
    k = 1024
    a, w = ints((m, k), 50 + m), ints((n, k), 51)
    g = torch.Generator().manual_seed(52)
    sa = (torch.rand((m, 1), generator=g) * 1e-2 + 1e-3).cuda()
    sb = (torch.rand((n, 1), generator=g) * 1e-3 + 1e-4).cuda()
    bias = torch.randn(n, generator=g).to(dtype).cuda()
    got = w8a8_mm(a, w.t(), sa, sb, dtype, bias)
    want = to_bits(og.epilogue_f32(exact(a, w), np_(sa), np_(sb), np_(bias)),
                   "bf16" if dtype == torch.bfloat16 else "f32")
    assert np.array_equal(bits(got), want)


def test_empty_batch():
    out = w8a8_mm(ints((0, 2048), 1), ints((64, 2048), 2).t(), one(), one())
    assert out.shape == (0, 64)


def test_choose_config_is_per_shape():
    decode, prefill = choose_config(1, 4096, 2048), choose_config(4096, 4096, 2048)
    assert decode.swapped or decode.split in (3, 5)   # swap_ab, narrow or CUDA-core decode tiles
    assert not prefill.swapped and prefill.split != 3


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("m,k,n", [(1, 2048, 2048), (37, 1024, 1000), (300, 512, 4096)])
def test_dequant_i32_equals_the_gemm_epilogue(dtype, m, k, n):
    """The standalone epilogue on an int32 product (the row-parallel path) equals the
    fused GEMM bit for bit."""
    from int8_linear.kernel import dequant_i32

    a, w = ints((m, k), 60), ints((n, k), 61)
    g = torch.Generator().manual_seed(62)
    sa = (torch.rand((m, 1), generator=g) * 1e-2 + 1e-3).cuda()
    sb = (torch.rand((n, 1), generator=g) * 1e-3 + 1e-4).cuda()
    bias = torch.randn(n, generator=g).to(dtype).cuda()
    acc = w8a8_mm(a, w.t(), one(), one(), raw=True)
    got = dequant_i32(acc, sa, sb, dtype, bias)
    assert torch.equal(got, w8a8_mm(a, w.t(), sa, sb, dtype, bias))


def test_out_argument_writes_in_place_with_the_same_bits():
    """`out=`: the product written into a given tensor (a slice of a larger buffer
    here) equals the returned one; a tensor of the wrong shape or dtype is refused."""
    m, k, n = 5, 2048, 1024
    a, w = ints((m, k), 400), ints((n, k), 401)
    g = torch.Generator().manual_seed(402)
    sa = (torch.rand((m, 1), generator=g) * 1e-2).cuda()
    sb = (torch.rand((n, 1), generator=g) * 1e-3).cuda()
    want = w8a8_mm(a, w.t(), sa, sb, torch.bfloat16)
    buf = torch.full((3 * m * n,), float("nan"), dtype=torch.bfloat16, device="cuda")
    out = buf[m * n: 2 * m * n].view(m, n)
    got = w8a8_mm(a, w.t(), sa, sb, torch.bfloat16, out=out)
    assert got.data_ptr() == out.data_ptr()
    assert np.array_equal(bits(out), bits(want))
    assert torch.isnan(buf[:m * n].float()).all() and torch.isnan(buf[2 * m * n:].float()).all()
    raw = torch.empty((m, n), dtype=torch.int32, device="cuda")
    w8a8_mm(a, w.t(), sa, sb, raw=True, out=raw)
    assert np.array_equal(np_(raw), exact(a, w))
    with pytest.raises(ValueError, match="out must be"):
        w8a8_mm(a, w.t(), sa, sb, torch.bfloat16, out=torch.empty((m, n), device="cuda"))


@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("k,n", [(1040, 1000), (1536, 256), (6144, 8192), (2048, 100)])
def test_untuned_one_and_two_token_batches_take_cuda_core_tiles_bit_exact(m, k, n):
    """Shapes missing from the tuned table fall to default_config, which sends one- and
    two-token batches to CUDA-core tiles: exact like every tiling."""
    from int8_linear.kernel import default_config, tuned_config

    assert tuned_config(m, n, k) is None
    cfg = default_config(m, n, k)
    assert cfg.split == 5 and cfg.bm >= m
    a, w = ints((m, k), 700 + m), ints((n, k), 701)
    g = torch.Generator().manual_seed(702)
    sa = (torch.rand((m, 1), generator=g) * 1e-2 + 1e-3).cuda()
    sb = (torch.rand((n, 1), generator=g) * 1e-3 + 1e-4).cuda()
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16).cuda()
    want = exact(a, w)
    assert np.array_equal(np_(w8a8_mm(a, w.t(), one(), one(), raw=True)), want)
    got = w8a8_mm(a, w.t(), sa, sb, torch.bfloat16, bias)
    assert np.array_equal(bits(got), to_bits(og.epilogue_f32(want, np_(sa), np_(sb), np_(bias)), "bf16"))


GEMV_SHAPES = [(16, 1), (48, 77), (2048, 4096), (6144, 2048), (2048, 12288), (14336, 4096), (1040, 1000),
               (4096, 28672)]


@pytest.mark.parametrize("m", [1, 2, 3, 5, 8, 13, 16])
@pytest.mark.parametrize("k,n", GEMV_SHAPES)
def test_cuda_core_tiles_bit_exact(m, k, n):
    """CUDA-core tiles (split 5): whole output columns per CTA, dp4a dot products; the
    int32 product exact and every output dtype bit-exact against the fp32 epilogue."""
    a, w = ints((m, k), 90 + m), ints((n, k), 91 + k)
    g = torch.Generator().manual_seed(92)
    sa = (torch.rand((m, 1), generator=g) * 1e-2 + 1e-3).cuda()
    sb = (torch.rand((n, 1), generator=g) * 1e-3 + 1e-4).cuda()
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16).cuda()
    cfg = Config(next(t for t in (1, 2, 4, 8, 16) if t >= m), 0, split=5)
    want = exact(a, w)
    if m * k > 200_000:   # the M x K activation and one ring stage exceed shared memory
        with pytest.raises(NotSupported, match="shared memory"):
            w8a8_mm(a, w.t(), one(), one(), raw=True, config=cfg)
        return
    assert np.array_equal(np_(w8a8_mm(a, w.t(), one(), one(), raw=True, config=cfg)), want)
    for dt, code in ((torch.bfloat16, "bf16"), (torch.float16, "f16"), (torch.float32, "f32")):
        got = w8a8_mm(a, w.t(), sa, sb, dt, bias, config=cfg)
        assert np.array_equal(bits(got), to_bits(og.epilogue_f32(want, np_(sa), np_(sb), np_(bias)), code)), dt


@pytest.mark.parametrize("cfg", [Config(8, 0, split=5, ctas=1), Config(4, 0, split=5, ctas=7),
                                 Config(8, 0, split=5, ctas=300), Config(2, 0, split=5, stages=1),
                                 Config(4, 0, split=5, stages=2), Config(8, 0, split=5, stages=3, ctas=37),
                                 Config(16, 0, split=5), Config(16, 0, split=5, ctas=296, stages=2)],
                         ids=lambda c: c.name)
def test_cuda_core_tiles_under_other_grids(cfg):
    """Fewer and more CTAs than SMs (each owning a contiguous column range) and short rings
    (stages refilled many times): same bits."""
    m, k, n = min(cfg.bm, 3), 6144, 4100
    a, w = ints((m, k), 93), ints((n, k), 94)
    got = w8a8_mm(a, w.t(), one(), one(), raw=True, config=cfg)
    assert np.array_equal(np_(got), exact(a, w))


def test_cuda_core_tiles_on_strided_operands():
    """A weight and an activation that are column slices of wider buffers (row strides
    larger than K: one bulk copy per weight row) and an output with a wider row stride."""
    m, k, n = 5, 2048, 1000
    a_full, w_full = ints((m, k + 64), 95), ints((n, k + 32), 96)
    a, w = a_full[:, :k], w_full[:, :k]
    out_full = torch.full((m, n + 8), float("nan"), dtype=torch.bfloat16, device="cuda")
    out = out_full[:, :n]
    sa, sb = torch.full((m, 1), 1e-2, device="cuda"), torch.full((n, 1), 1e-3, device="cuda")
    w8a8_mm(a, w.t(), sa, sb, torch.bfloat16, config=Config(8, 0, split=5), out=out)
    want = exact(a.contiguous(), w.contiguous())
    assert np.array_equal(bits(out), to_bits(og.epilogue_f32(want, np_(sa), np_(sb)), "bf16"))
    assert bool(out_full[:, n:].isnan().all())    # nothing written past the rows


def test_cuda_core_tiles_decline_larger_batches():
    with pytest.raises(NotSupported):
        w8a8_mm(ints((9, 2048), 1), ints((64, 2048), 2).t(), one(), one(), config=Config(8, 0, split=5))
    with pytest.raises(NotSupported):
        w8a8_mm(ints((17, 2048), 1), ints((64, 2048), 2).t(), one(), one(), config=Config(16, 0, split=5))


@pytest.mark.parametrize("m", [65, 100, 128, 200, 256])
@pytest.mark.parametrize("k,n", [(2048, 4096), (6144, 2048), (2048, 12288), (1040, 1000)])
@pytest.mark.parametrize("cluster", [2, 3, 4, 8])
@pytest.mark.parametrize("store", [0, 1])
def test_cluster_split_wide_token_tiles(m, k, n, cluster, store):
    """Cluster split-K on 128- and 256-token swap tiles: each CTA finishes the 16-column
    chunks c with c % cluster == its rank from the others' partial sums (ragged last
    chunks when M is not a multiple of 16, ranks that own no live chunk)."""
    a, w = ints((m, k), 100 + m), ints((n, k), 101)
    g = torch.Generator().manual_seed(102)
    sa = (torch.rand((m, 1), generator=g) * 1e-2 + 1e-3).cuda()
    sb = (torch.rand((n, 1), generator=g) * 1e-3 + 1e-4).cuda()
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16).cuda()
    cfg = Config(tok_tile(m), 128, swap_ab=True, split=3, cluster=cluster, store=store)
    want = exact(a, w)
    if tok_tile(m) == 256 and cluster == 8:   # 7 x 2 chunks in + 14 out: 224 KB > the 192 KB ring
        with pytest.raises(NotSupported, match="ring"):
            w8a8_mm(a, w.t(), one(), one(), raw=True, config=cfg)
        return
    got = w8a8_mm(a, w.t(), one(), one(), raw=True, config=cfg)
    assert np.array_equal(np_(got), want)
    got = w8a8_mm(a, w.t(), sa, sb, torch.bfloat16, bias, config=cfg)
    assert np.array_equal(bits(got), to_bits(og.epilogue_f32(want, np_(sa), np_(sb), np_(bias)), "bf16"))


@pytest.mark.parametrize("m", [65, 128, 200, 256])
@pytest.mark.parametrize("k,n", [(6144, 256), (2048, 512), (14336, 512), (4096, 768), (6144, 1536), (2048, 256)])
def test_default_tiles_of_untuned_shapes(m, k, n):
    """Tensor-parallel shards and other shapes outside the tile table take the library's
    own choice (cluster split-K sized to fit the ring for 128/256-token tiles on few
    tiles): it must run and be exact."""
    a, w = ints((m, k), 300 + m), ints((n, k), 301)
    assert np.array_equal(np_(w8a8_mm(a, w.t(), one(), one(), raw=True)), exact(a, w))

