"""Seeded CPU input recipes shared by make_golden.py and the tests.

Each follows a reference test's or benchmark's input generation (AshrithaG/int8-linear),
with torch's CPU generator in place of its CUDA one, so the inputs can be rebuilt
anywhere bit for bit; the golden manifest stores a SHA-256 of each input to prove it.
"""

from __future__ import annotations

import hashlib

import numpy as np
import torch

EPS = 1e-6
# (M, K, N) of tests/test_kernel.py:22
GEMM_SHAPES = [(1, 2048, 2048), (3, 2048, 1024), (17, 2048, 6144), (64, 2048, 2048), (100, 6144, 2048)]
# tests/test_fused_quant.py:64 and :78
NORM_SHAPES = [(1, 2048), (7, 2048), (64, 1024), (300, 2048), (5, 1000)]
SILU_SHAPES = [(1, 6144), (33, 6144), (8, 1000)]


def sha(t) -> str:
    if isinstance(t, torch.Tensor):
        t = t.contiguous()
        if t.dtype == torch.bfloat16:
            t = t.view(torch.int16)
        t = t.numpy()
    return hashlib.sha256(np.ascontiguousarray(t).tobytes()).hexdigest()


def config0():
    """A bf16 N(0,1) [16, 2048], W bf16 N(0, 0.02) [2048, 2048],
    drawn in that order from one generator seeded 0 (bench/bench_linear.py:153-156)."""
    g = torch.Generator().manual_seed(0)
    a = torch.randn((16, 2048), generator=g).to(torch.bfloat16)
    w = (torch.randn((2048, 2048), generator=g) * 0.02).to(torch.bfloat16)
    return a, w


def ints(shape, seed):
    """tests/test_kernel.py:25-27 on a CPU generator."""
    g = torch.Generator().manual_seed(seed)
    return torch.randint(-127, 128, shape, dtype=torch.int8, generator=g)


def scaled_case(dtype, per_row, per_col, use_bias):
    """Operands of tests/test_kernel.py:60-66."""
    m, k, n = 37, 2048, 1024
    a, w = ints((m, k), 5), ints((n, k), 6)
    g = torch.Generator().manual_seed(7)
    sa = torch.rand((m, 1) if per_row else (1,), generator=g) * 1e-2 + 1e-3
    sb = torch.rand((n, 1) if per_col else (1,), generator=g) * 1e-2 + 1e-3
    bias = torch.randn(n, generator=g).to(dtype) if use_bias else None
    return a, w, sa, sb, bias


def rand(shape, seed, scale=1.0, dtype=torch.bfloat16):
    """tests/test_fused_quant.py:19-21 on a CPU generator."""
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(dtype)


def norm_case(m, k, has_res):
    """Operands of tests/test_fused_quant.py:64-75."""
    x = rand((m, k), m)
    r = rand((m, k), m + 1) if has_res else None
    w = rand((k,), 99, 0.1) + 1.0
    return x, r, w


def silu_case(m, i):
    """Operands of tests/test_fused_quant.py:78-83."""
    return rand((m, 2 * i), m, 2.0)


def outlier_activations(m, k, seed):
    """bench/fuse_quant.py:52-57 on a CPU generator: N(0,1) with 8 channels x30."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((m, k), generator=g)
    x[:, torch.randperm(k, generator=g)[:8]] *= 30.0
    return x.to(torch.bfloat16)
