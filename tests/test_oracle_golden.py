"""The oracle against the reference's own outputs (tests/golden, made by
tests/golden/make_golden.py from the reference's functions).  CPU only."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import gemm as og
from oracle import quant as oq
from oracle.numerics import f32_to_bf16_bits, round_bf16
from tests.golden import recipes

GOLDEN = Path(__file__).resolve().parent / "golden"
MAN = json.loads((GOLDEN / "golden.json").read_text())["cases"]
ARR = np.load(GOLDEN / "golden.npz")


def f32(t: torch.Tensor) -> np.ndarray:
    return t.float().numpy()


def test_config0_operands_and_product():
    x, w = recipes.config0()
    case = MAN["config0"]
    assert recipes.sha(x) == case["x"] and recipes.sha(w) == case["w"]  # same inputs
    a_q, a_s = og.quant_rows(f32(x))
    w_q, w_s = og.quant_rows(f32(w))
    assert np.array_equal(a_q, ARR["c0_a_q"]) and np.array_equal(a_s, ARR["c0_a_s"])
    assert np.array_equal(w_s, ARR["c0_w_s"]) and recipes.sha(w_q) == case["w_q"]
    acc = og.exact(a_q, w_q)
    assert recipes.sha(acc) == case["acc"]
    term, ref = og.scaled_ref(acc, a_s, w_s)
    assert recipes.sha(ref) == case["ref"]
    # the fp32 epilogue lands within one bf16 step of the float64 layer rounded to bf16
    bits = f32_to_bf16_bits(og.epilogue_f32(acc, a_s, w_s)).astype(np.int32)
    assert np.abs(bits - ARR["c0_ref_bf16"].astype(np.int32)).max() <= 1
    assert og.rel_error(round_bf16(og.epilogue_f32(acc, a_s, w_s)), term, ref) < 1e-2


@pytest.mark.parametrize("m,k,n", recipes.GEMM_SHAPES)
def test_exact_products(m, k, n):
    a, w = recipes.ints((m, k), 1), recipes.ints((n, k), 2)
    case = MAN[f"exact_{m}x{k}x{n}"]
    assert recipes.sha(a) == case["a"] and recipes.sha(w) == case["w"]
    out = og.exact(a.numpy(), w.numpy())
    assert recipes.sha(out) == case["out"]
    if f"exact_{m}x{k}x{n}" in ARR:
        assert np.array_equal(out, ARR[f"exact_{m}x{k}x{n}"])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("per_row", [True, False])
@pytest.mark.parametrize("per_col", [True, False])
@pytest.mark.parametrize("use_bias", [True, False])
def test_scaled_layer(dtype, per_row, per_col, use_bias):
    a, w, sa, sb, bias = recipes.scaled_case(dtype, per_row, per_col, use_bias)
    case = MAN[f"scaled_{str(dtype)[6:]}_{int(per_row)}{int(per_col)}{int(use_bias)}"]
    acc = og.exact(a.numpy(), w.numpy())
    term, ref = og.scaled_ref(acc, sa.numpy(), sb.numpy(), f32(bias) if use_bias else None)
    assert recipes.sha(term) == case["term"] and recipes.sha(ref) == case["ref"]
    got = og.epilogue_f32(acc, sa.numpy(), sb.numpy(), f32(bias) if use_bias else None)
    rounded = round_bf16(got) if dtype == torch.bfloat16 else got.astype(np.float16).astype(np.float32)
    assert og.rel_error(rounded, term, ref) < 1e-2


@pytest.mark.parametrize("m,k", recipes.NORM_SHAPES)
@pytest.mark.parametrize("has_res", [False, True])
def test_norm_quant(m, k, has_res):
    x, r, w = recipes.norm_case(m, k, has_res)
    key = f"norm_{m}x{k}_{int(has_res)}"
    assert recipes.sha(x) == MAN[key]["x"] and recipes.sha(w) == MAN[key]["w"]
    q, s, rout = oq.ref_norm(f32(x), f32(r) if has_res else None, f32(w), recipes.EPS)
    d = oq.compare_int8(q, s, ARR[key + "_q"], ARR[key + "_s"])
    assert d.count == 0 and d.scale_rel == 0, d     # bit-exact with the reference's ref_norm
    if has_res:
        assert recipes.sha(f32_to_bf16_bits(rout).view(np.int16)) == MAN[key]["rout"]


@pytest.mark.parametrize("m,i", recipes.SILU_SHAPES)
@pytest.mark.parametrize("rnd", [False, True])
def test_silu_quant(m, i, rnd):
    gu = recipes.silu_case(m, i)
    key = f"silu_{m}x{i}_{int(rnd)}"
    assert recipes.sha(gu) == MAN[key]["gu"]
    q, s = oq.ref_silu(f32(gu), rnd)
    d = oq.compare_int8(q, s, ARR[key + "_q"], ARR[key + "_s"])
    assert d.count == 0 and d.scale_rel == 0, d     # bit-exact with the reference's ref_silu


def test_plain_quant_is_bit_exact():
    x = recipes.outlier_activations(64, 2048, 5)
    assert recipes.sha(x) == MAN["outlier_64x2048"]["x"]
    q, s = oq.quant(f32(x))
    assert np.array_equal(q, ARR["outlier_q"]) and np.array_equal(s, ARR["outlier_s"])


def test_zero_row_and_saturation():
    q, s = oq.quant(np.zeros((3, 64), np.float32))
    assert not q.any() and not s.any()
    y = np.random.default_rng(0).standard_normal((16, 512)).astype(np.float32)
    q, _ = oq.quant(y)
    assert (np.abs(q.astype(np.int32)).max(axis=1) == 127).all()


def test_compare_int8_catches_a_planted_error():
    """The checker itself: a planted two-step error and too many one-step errors fail."""
    q = np.zeros((4, 4096), np.int8)
    s = np.ones((4, 1), np.float32)
    bad = q.copy()
    bad[0, 0] = 2
    assert not oq.compare_int8(bad, s, q, s).ok()
    many = q.copy()
    many[:, :100] = 1
    assert not oq.compare_int8(many, s, q, s).ok()
    assert oq.compare_int8(q, s * (1 + 1e-4), q, s).scale_rel > 1e-5


@pytest.mark.parametrize("use_bias", [False, True])
def test_torch_float64_layer_is_the_numpy_layer(use_bias):
    """The torch restatement the benchmark times as the reference's CPU path
    (bench/bench_linear.py:164-165) gives the numpy oracle's float64 values, and its bf16
    output is the float64 layer rounded once."""
    a, w, sa, sb, bias = recipes.scaled_case(torch.bfloat16, True, True, use_bias)
    acc = og.exact(a.numpy(), w.numpy())
    _, ref = og.scaled_ref(acc, sa.numpy(), sb.numpy(), f32(bias) if use_bias else None)
    got64 = og.layer_f64_torch(a, sa.reshape(-1, 1), w, sb.reshape(-1, 1),
                               bias if use_bias else None, torch.float64)
    assert np.array_equal(got64.numpy(), ref)
    got = og.layer_f64_torch(a, sa.reshape(-1, 1), w, sb.reshape(-1, 1), bias if use_bias else None)
    assert torch.equal(got, torch.from_numpy(ref).to(torch.bfloat16))
