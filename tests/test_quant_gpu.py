"""The sm_100a fused quantisers against the CPU oracle (oracle/quant.py).

Mirrors the reference's tests/test_fused_quant.py (same shapes, the same tolerance:
|dq| <= 1, at most max(8, 1e-3 n) differing values, scales within 1e-5, residual
bit-identical) and reports how many values differ.  Against the oracle's restatement
of the kernel's own arithmetic (IEEE-divide quantiser) the SiLU and plain
quantisers are bit-exact; the norm differs only where the sum of squares is reduced
in another order.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from int8_linear import fused_quant as fq
from int8_linear import vllm_fuse_patch as vfp
from oracle import quant as oq
from oracle.numerics import f32_to_bf16_bits
from tests.gpu_util import bits, np_, rand

pytestmark = pytest.mark.gpu
EPS = 1e-6
DT = {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}


def check(q, s, q_ref, s_ref, exact=False):
    d = oq.compare_int8(np_(q), np_(s), q_ref, s_ref)
    assert d.ok(), d
    if exact:
        assert d.count == 0 and d.scale_rel == 0, d
    return d


@pytest.mark.parametrize("m,k", [(1, 2048), (7, 2048), (64, 1024), (300, 2048), (5, 1000),
                                 (4096, 2048), (3, 4096), (2, 14336), (9, 8)])
@pytest.mark.parametrize("has_res", [False, True])
def test_add_rmsnorm_quant(m, k, has_res):
    x = rand((m, k), m)
    r = rand((m, k), m + 1) if has_res else None
    w = rand((k,), 99, 0.1) + 1.0
    q, s, rout = fq.add_rmsnorm_quant(x, r, w, EPS, precise_div=True)
    assert q.dtype == torch.int8 and s.shape == (m, 1)
    xr, rr, wr = np_(x), np_(r) if has_res else None, np_(w)
    check(q, s, *oq.ref_norm(xr, rr, wr, EPS)[:2])                                # reference tolerance
    check(q, s, *oq.ref_norm(xr, rr, wr, EPS, quantiser=oq.quant_ieee)[:2])        # kernel arithmetic
    if has_res:
        _, _, r0 = oq.ref_norm(xr, rr, wr, EPS)
        assert np.array_equal(bits(rout), f32_to_bf16_bits(r0))                    # residual exact


@pytest.mark.parametrize("act", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("wdt", [torch.bfloat16, torch.float16, torch.float32])
def test_add_rmsnorm_quant_dtypes(act, wdt):
    m, k = 33, 2048
    x, r = rand((m, k), 1, dtype=act), rand((m, k), 2, dtype=act)
    w = (rand((k,), 3, 0.1, torch.float32) + 1.0).to(wdt)
    q, s, rout = fq.add_rmsnorm_quant(x, r, w, EPS)
    q0, s0, r0 = oq.ref_norm(np_(x), np_(r), np_(w), EPS, act=DT[act], wdt=DT[wdt],
                             quantiser=oq.quant_ieee, kernel_order=True)
    check(q, s, q0, s0)
    assert np.array_equal(np_(rout), r0)


@pytest.mark.parametrize("m,i", [(1, 6144), (33, 6144), (8, 1000), (4096, 6144), (2, 14336)])
@pytest.mark.parametrize("round_silu", [False, True])
def test_silu_mul_quant(m, i, round_silu):
    gu = rand((m, 2 * i), m, 2.0)
    q, s = fq.silu_mul_quant(gu, precise_div=True, round_silu=round_silu)
    check(q, s, *oq.ref_silu(np_(gu), round_silu))
    check(q, s, *oq.ref_silu(np_(gu), round_silu, quantiser=oq.quant_ieee))


@pytest.mark.parametrize("m,k", [(1, 2048), (64, 2048), (7, 1000), (4096, 4096)])
def test_per_token_quant(m, k):
    x = rand((m, k), m + k, 3.0)
    q, s = fq.per_token_quant(x)
    check(q, s, *oq.quant(np_(x)))
    check(q, s, *oq.quant_ieee(np_(x)), exact=True)


def test_per_token_quant_on_a_column_slice():
    """The stand-in decoder quantises qkv[:, :2048] in place, without a copy."""
    qkv = rand((17, 4096), 4)
    q, s = fq.per_token_quant(qkv[:, :2048])
    check(q, s, *oq.quant_ieee(np_(qkv)[:, :2048]), exact=True)


def test_approximate_division_stays_within_tolerance():
    gu = rand((64, 2 * 6144), 9, 2.0)
    q, s = fq.silu_mul_quant(gu, precise_div=False)
    check(q, s, *oq.ref_silu(np_(gu), False))


def test_zero_row_gives_zero_scale_and_values():
    x = torch.zeros((3, 2048), device="cuda", dtype=torch.bfloat16)
    w = torch.ones(2048, device="cuda", dtype=torch.bfloat16)
    q, s, _ = fq.add_rmsnorm_quant(x, None, w, EPS)
    assert q.abs().max().item() == 0 and s.abs().max().item() == 0
    q, s = fq.per_token_quant(x)
    assert q.abs().max().item() == 0 and s.abs().max().item() == 0


def test_saturates_at_127():
    """The largest-magnitude element of every row lands on +-127 exactly."""
    gu = rand((16, 2 * 512), 5, 3.0)
    q, _ = fq.silu_mul_quant(gu)
    assert q.int().abs().amax(-1).eq(127).all()


def test_empty_batch():
    q, s, r = fq.add_rmsnorm_quant(rand((0, 2048), 1), rand((0, 2048), 2),
                                   torch.ones(2048, device="cuda", dtype=torch.bfloat16), EPS)
    assert q.shape == (0, 2048) and s.shape == (0, 1) and r.shape == (0, 2048)


def test_custom_ops_opcheck():
    x, r = rand((9, 2048), 1), rand((9, 2048), 2)
    w = rand((2048,), 3) + 1.0
    torch.library.opcheck(fq.rmsnorm_quant_op, (x, w, EPS))
    torch.library.opcheck(fq.add_rmsnorm_quant_op, (x, r, w, EPS))
    torch.library.opcheck(fq.silu_mul_quant_op, (rand((9, 2 * 6144), 4),))
    torch.library.opcheck(fq.per_token_quant_op, (x,))


def test_prequant_matmul_matches_unfused():
    """What the fuse patch feeds down_proj equals quantising silu's output then the GEMM."""
    from int8_linear import w8a8_mm
    from tests.gpu_util import ints

    gu = rand((5, 2 * 6144), 6, 2.0)
    q, s = fq.silu_mul_quant(gu)
    w = ints((2048, 6144), 7)
    ws = torch.rand((2048, 1), device="cuda") * 1e-3 + 1e-4
    pq = vfp.PreQuant(q, s, torch.bfloat16)
    out = w8a8_mm(pq.data, w.t(), pq.scale, ws, pq.dtype)
    assert out.shape == (5, 2048) and torch.isfinite(out.float()).all()


@pytest.mark.parametrize("m,k", [(1, 2048), (33, 1024), (7, 1000)])
def test_split_row_quantisation_with_a_given_absmax(m, k):
    """row_absmax / silu_mul_absmax and quantising with a given absmax (the pieces of a
    row split across GPUs) reproduce the whole-row quantiser."""
    x = rand((m, k), 40, 3.0)
    amax = fq.row_absmax(x)
    assert torch.equal(amax, np_t(x).abs().amax(-1))
    q, s = fq.per_token_quant(x, absmax=amax)
    q0, s0 = fq.per_token_quant(x)
    assert torch.equal(q, q0) and torch.equal(s, s0)
    # a larger absmax (another GPU's half of the row) scales the same way the oracle does
    big = amax * 1.5
    q, s = fq.per_token_quant(x, absmax=big)
    qo, so = oq.quant_ieee(np_(x), np_(big))
    check(q, s, qo, so, exact=True)
    gu = rand((m, 2 * k), 41, 2.0)
    amax = fq.silu_mul_absmax(gu, round_silu=True)
    q, s = fq.silu_mul_quant(gu, True, True, absmax=amax)
    q0, s0 = fq.silu_mul_quant(gu, True, True)
    assert torch.equal(q, q0) and torch.equal(s, s0)
    # scale = absmax / 127 with an IEEE divide (numpy's float32 division)
    assert np.array_equal(np_(s).reshape(-1), (np_(amax) / np.float32(127.0)).astype(np.float32))


def np_t(x):
    return x.float()


@pytest.mark.parametrize("kind", ["silu", "plain"])
@pytest.mark.parametrize("m,cols", [(1, 6144), (5, 6144), (3, 14336), (17, 4096), (9, 3080), (2, 12296)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_decode_batch_rows_equal_large_batch_rows(kind, m, cols, dtype):
    """A decode batch (fewer rows than SMs) spreads each row over up to 1024 threads; the
    same rows inside a batch of 200 use 256-thread CTAs.  The row reduction is a maximum,
    so both give the same bits."""
    g = torch.Generator().manual_seed(m * 13 + cols)
    width = 2 * cols if kind == "silu" else cols
    big = (torch.randn((200, width), generator=g) * 3).to(dtype).cuda()
    small = big[:m].contiguous()
    if kind == "silu":
        for rs in (False, True):
            q0, s0 = fq.silu_mul_quant(big, True, rs)
            q1, s1 = fq.silu_mul_quant(small, True, rs)
            assert torch.equal(q1, q0[:m]) and torch.equal(s1, s0[:m])
    else:
        q0, s0 = fq.per_token_quant(big)
        q1, s1 = fq.per_token_quant(small)
        assert torch.equal(q1, q0[:m]) and torch.equal(s1, s0[:m])
        xs = big[:m, 4:cols - 4]           # an unaligned slice takes the scalar path
        q2, s2 = fq.per_token_quant(xs)
        qo, so = oq.quant_ieee(np_(xs))
        check(q2, s2, qo, so, exact=True)


@pytest.mark.parametrize("m,k", [(2049, 2048), (4096, 2048), (2049, 4096), (2048, 8192), (2048, 1000)])
@pytest.mark.parametrize("act,wdt", [(torch.bfloat16, torch.bfloat16), (torch.float16, torch.float32)])
def test_large_batch_norm_rows_equal_small_batch_rows(m, k, act, wdt):
    """Large batches normalise two rows per CTA (odd batches end with a one-row CTA); each
    row's arithmetic is the one-row kernel's, so rows agree bit for bit with the same rows
    in a small batch, residual output included."""
    x, r = rand((m, k), 500 + m, dtype=act), rand((m, k), 501 + m, dtype=act)
    w = (rand((k,), 502, 0.1, torch.float32) + 1.0).to(wdt)
    q0, s0, r0 = fq.add_rmsnorm_quant(x, r, w, EPS)
    for lo, hi in ((0, 5), (m - 3, m)):
        q1, s1, r1 = fq.add_rmsnorm_quant(x[lo:hi].contiguous(), r[lo:hi].contiguous(), w, EPS)
        assert torch.equal(q1, q0[lo:hi]) and torch.equal(s1, s0[lo:hi]), (lo, hi)
        assert np.array_equal(bits(r1), bits(r0[lo:hi]))
    q2, s2, _ = fq.add_rmsnorm_quant(x, None, w, EPS)
    q3, s3, _ = fq.add_rmsnorm_quant(x[-3:].contiguous(), None, w, EPS)
    assert torch.equal(q3, q2[-3:]) and torch.equal(s3, s2[-3:])
