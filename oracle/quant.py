"""Oracle for the fused per-token int8 quantisers (numpy).  Test infrastructure only.

Restates, from the reference AshrithaG/int8-linear:
  quant            tests/test_fused_quant.py:26-31  (torch's arithmetic, round half even)
  quant_ieee       int8_linear/fused_quant.py:41-53 (the kernel's IEEE-divide quantiser)
  ref_norm         tests/test_fused_quant.py:34-42  (add + RMSNorm, then quant)
  ref_silu         tests/test_fused_quant.py:45-51  (SiLU-and-mul, then quant)
  compare_int8     tests/test_fused_quant.py:54-61  (the reference's tolerance:
                   |dq| <= 1, at most max(8, 1e-3 n) differing values, scales within
                   1e-5 relative), extended to report the differing count.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from oracle.numerics import round_to


def quant(y: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """The reference's torch `quant` (tests/test_fused_quant.py:26-31), step for step:
    absmax = max|y|; inv = 127.0 / absmax, which torch evaluates as
    reciprocal(absmax) * 127 (Tensor.__rtruediv__, two float32 roundings) and 0 where
    absmax == 0; q = clamp(round_half_even(y * inv), -128, 127); scale = absmax / 127
    (a true float32 division)."""
    yf = np.asarray(y, dtype=np.float32)
    absmax = np.abs(yf).max(axis=-1, keepdims=True)
    with np.errstate(divide="ignore"):
        recip = (np.float32(1.0) / absmax).astype(np.float32)
    inv = np.where(absmax == 0, np.float32(0), recip * np.float32(127.0)).astype(np.float32)
    q = np.clip(np.rint(yf * inv), -128, 127).astype(np.int8)
    return q, (absmax / np.float32(127.0)).astype(np.float32)


def quant_ieee(y: np.ndarray, absmax: np.ndarray | None = None) -> tuple[np.ndarray, np.ndarray]:
    """The reference KERNEL's row quantiser with precise_div (int8_linear/fused_quant.py:
    41-53): inv = div_rn(127, absmax), one IEEE rounding; otherwise as `quant`.  A given
    `absmax` (one per row) replaces the row's own, as for a row split across GPUs."""
    yf = np.asarray(y, dtype=np.float32)
    if absmax is None:
        absmax = np.abs(yf).max(axis=-1, keepdims=True)
    else:
        absmax = np.asarray(absmax, np.float32).reshape(-1, 1)
    with np.errstate(divide="ignore"):
        inv = np.where(absmax == 0, np.float32(0), np.float32(127.0) / absmax).astype(np.float32)
    q = np.clip(np.rint(yf * inv), -128, 127).astype(np.int8)
    return q, (absmax / np.float32(127.0)).astype(np.float32)


def ref_norm(x: np.ndarray, r: np.ndarray | None, w: np.ndarray, eps: float,
             act: str = "bf16", wdt: str = "bf16", quantiser=None, kernel_order: bool = False):
    """(q, scale, residual_out) for add + RMSNorm + quant.  x, r, w are float32 arrays
    holding act/wdt values.  residual_out is float32 holding act values, or None.

    The product with the weight: torch (the reference's ref_norm) rounds it to the
    weight dtype and then to the activation dtype; the reference kernel
    (int8_linear/fused_quant.py:72) rounds the fp32 product once, to the activation
    dtype (kernel_order=True).  The two agree whenever the weight dtype is the
    activation dtype or float32."""
    xf = np.asarray(x, dtype=np.float32)
    rout = None
    if r is not None:
        xf = (xf + np.asarray(r, dtype=np.float32)).astype(np.float32)
        rout = round_to(xf, act)
    var = (np.sum(xf.astype(np.float64) ** 2, axis=-1, keepdims=True) / xf.shape[-1]).astype(np.float32)
    rs = (np.float32(1.0) / np.sqrt((var + np.float32(eps)).astype(np.float32))).astype(np.float32)
    xn = round_to((xf * rs).astype(np.float32), wdt)
    prod = (xn * np.asarray(w, np.float32)).astype(np.float32)
    y = round_to(prod if kernel_order else round_to(prod, wdt), act)
    q, s = (quantiser or quant)(y)
    return q, s, rout


def ref_silu(gu: np.ndarray, round_silu: bool, act: str = "bf16", quantiser=None):
    """(q, scale) for silu(gate) * up then quant; gate = first half of each row."""
    gu = np.asarray(gu, dtype=np.float32)
    i = gu.shape[1] // 2
    g, u = gu[:, :i], gu[:, i:]
    a = (g / (np.float32(1.0) + np.exp(-g, dtype=np.float32))).astype(np.float32)
    if round_silu:
        a = round_to(a, act)
    return (quantiser or quant)(round_to((a * u).astype(np.float32), act))


@dataclass
class Int8Diff:
    max_abs: int        # largest |q - q_ref|
    count: int          # values that differ
    numel: int
    scale_rel: float    # largest relative scale difference

    @property
    def allowed(self) -> int:
        return max(8, int(1e-3 * self.numel))

    def ok(self) -> bool:
        return self.max_abs <= 1 and self.count <= self.allowed and self.scale_rel < 1e-5


def compare_int8(q, s, q_ref, s_ref) -> Int8Diff:
    """The reference's assert_close_int8 measure, returned instead of asserted."""
    d = np.abs(np.asarray(q, np.int32) - np.asarray(q_ref, np.int32))
    s, s_ref = np.asarray(s, np.float64), np.asarray(s_ref, np.float64)
    rel = np.abs(s - s_ref) / np.maximum(np.abs(s_ref), 1e-30)
    return Int8Diff(int(d.max(initial=0)), int((d != 0).sum()), int(d.size),
                    float(rel.max(initial=0.0)))
