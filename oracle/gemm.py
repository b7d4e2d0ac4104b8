"""Oracle for the W8A8 GEMM (numpy).  Test infrastructure only (oracle/__init__.py).

Restates, from the reference AshrithaG/int8-linear:
  quant_rows         bench/bench_linear.py:146-150  (operand generation)
  exact              tests/test_kernel.py:36-38     (exact int32 product)
  scaled_ref         bench/bench_linear.py:164-165, tests/test_kernel.py:68-69
                     (the float64 quantised layer)
  epilogue_f32       int8_linear/kernel.py:109-120  (the kernel's fp32 epilogue
                     order: f32(acc) * sa, * sb, + f32(bias), one rounding)
  rel_error          tests/test_kernel.py:70-75, bench/bench_linear.py:190-192
"""

from __future__ import annotations

import numpy as np

from oracle.numerics import to_bits


def quant_rows(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Symmetric int8 with one float32 scale per row (bench_linear.py:146-150):
    scale = max|x| (at least 1e-8) / 127, q = round_half_even(x / scale) clamped to
    +-127.  x is float32 [R, C]; returns (int8 [R, C], float32 [R, 1])."""
    xf = np.asarray(x, dtype=np.float32)
    amax = np.maximum(np.abs(xf).max(axis=1, keepdims=True), np.float32(1e-8))
    scale = (amax / np.float32(127.0)).astype(np.float32)
    q = np.clip(np.rint(xf / scale), -127, 127).astype(np.int8)
    return q, scale


def exact(a_q: np.ndarray, w_q: np.ndarray) -> np.ndarray:
    """A_q [M, K] @ W_q[N, K]^T as int32 (test_kernel.py:36-38).  A float64 product of
    int8 values is exact (every partial sum < 2**53), so BLAS order does not matter."""
    return (a_q.astype(np.float64) @ w_q.astype(np.float64).T).astype(np.int32)


def scaled_ref(acc: np.ndarray, sa: np.ndarray, sb: np.ndarray,
               bias: np.ndarray | None = None) -> tuple[np.ndarray, np.ndarray]:
    """(term, ref) in float64: term = acc * sa[m] * sb[n]; ref = term + bias[n]
    (bench_linear.py:164-165; test_kernel.py:68-69).  sa is [M] or [1], sb [N] or [1]."""
    term = (acc.astype(np.float64) * np.asarray(sa, np.float64).reshape(-1, 1)
            * np.asarray(sb, np.float64).reshape(1, -1))
    ref = term + np.asarray(bias, np.float64).reshape(1, -1) if bias is not None else term
    return term, ref


def layer_f64_torch(a_q, a_s, w_q, w_s, bias=None, out_dtype=None):
    """The reference's float64 layer in torch, as bench/bench_linear.py:164-165 writes it:
    term = (A_q.double() @ W_q.double().t()) * a_s.double() * w_s.double().t(), plus
    bias.double(); rounded to out_dtype (bf16 unless given).  a_q int8 [M, K], a_s
    float32 [M, 1], w_q int8 [N, K], w_s float32 [N, 1], bias [N] or None, all torch
    CPU tensors.  This is the CPU path the benchmark times as the reference; its
    float64 values equal `scaled_ref` on the same inputs (tests/test_oracle_golden.py)."""
    import torch

    term = (a_q.double() @ w_q.double().t()) * a_s.double() * w_s.double().t()
    ref = term + bias.double() if bias is not None else term
    return ref.to(out_dtype or torch.bfloat16)


def epilogue_f32(acc: np.ndarray, sa: np.ndarray, sb: np.ndarray,
                 bias: np.ndarray | None = None) -> np.ndarray:
    """The kernel's epilogue in float32, each step rounded (kernel.py:109-120):
    ((f32(acc) * sa[m]) * sb[n]) + f32(bias[n]).  Returns float32 before the final
    rounding to the output dtype."""
    v = acc.astype(np.float32)
    v = v * np.asarray(sa, np.float32).reshape(-1, 1)
    v = v * np.asarray(sb, np.float32).reshape(1, -1)
    if bias is not None:
        v = v + np.asarray(bias, np.float32).reshape(1, -1)
    return v.astype(np.float32)


def w8a8_out_bits(acc, sa, sb, bias, out_dtype: str) -> np.ndarray:
    """The output tensor's storage bits for out_dtype in {'bf16','f16','f32'}."""
    return to_bits(epilogue_f32(acc, sa, sb, bias), out_dtype)


def rel_error(got: np.ndarray, term: np.ndarray, ref: np.ndarray) -> float:
    """max |got - ref| / max(|ref|, |term|, 1e-6) (test_kernel.py:70-75)."""
    scale = np.maximum(np.maximum(np.abs(ref), np.abs(term)), 1e-6)
    return float((np.abs(np.asarray(got, np.float64) - ref) / scale).max(initial=0.0))
