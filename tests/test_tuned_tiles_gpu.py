"""Every tiling the library picks at the benchmarked shapes, against the oracle.

w8a8_mm takes its tile from choose_config: the B200 table (int8_linear/tuned_configs.json)
or, for an untuned shape, default_config; bench.py times exactly these.  This walks every
shape of the table at every M of the sweep: BASELINE config 1 (Qwen3-1.7B as vLLM runs
it), config 2 (Llama-3-8B), and the tensor-parallel shards (column-parallel N/2, N/4,
N/8; row-parallel K/2, K/4, K/8).  For each it checks the int32 product bit for bit
against oracle.exact (tests/test_kernel.py:36-38 in the reference) and the bf16 output
with bias bit for bit against the fp32 epilogue restatement (int8_linear/kernel.py:
109-120), and within the reference's 1% of the float64 layer.  For M >= 256 the
check samples 24 rows (first, last and evenly spaced) to keep the CPU oracle in seconds.
"""

from __future__ import annotations

import json
from functools import lru_cache
from pathlib import Path

import numpy as np
import pytest
import torch

from int8_linear import w8a8_mm
from int8_linear.kernel import choose_config
from oracle import gemm as og
from oracle.numerics import to_bits
from tests.gpu_util import bits, ints, np_

pytestmark = pytest.mark.gpu

TABLE = json.loads((Path(__file__).resolve().parent.parent / "int8_linear" / "tuned_configs.json")
                   .read_text())["NVIDIA B200"]
M_SWEEP = [1, 2, 4, 8, 16, 17, 32, 64, 128, 256, 1024, 4096]
CASES = [(key, m) for key in sorted(TABLE, key=lambda s: tuple(map(int, s.split("x")))) for m in M_SWEEP]


@lru_cache(maxsize=2)
def weight(k: int, n: int):
    """One seeded int8 weight per shape (GPU), its float64 copy for the oracle, per-channel
    scales and a bias."""
    w = ints((n, k), k * 31 + n)
    g = torch.Generator().manual_seed(n)
    sb = torch.rand((n, 1), generator=g) * 1e-3 + 1e-4
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16)
    return w, np_(w).astype(np.float64), sb, bias


def sample_rows(m: int) -> np.ndarray:
    if m < 256:
        return np.arange(m)
    return np.unique(np.concatenate([[0, m - 1], np.linspace(0, m - 1, 22).astype(int)]))


@pytest.mark.parametrize("key,m", CASES, ids=[f"{k}-M{m}" for k, m in CASES])
def test_chosen_tile_is_exact(key, m):
    k, n = map(int, key.split("x"))
    w, w64, sb, bias = weight(k, n)
    a = ints((m, k), m * 7919 + k)
    g = torch.Generator().manual_seed(m)
    sa = torch.rand((m, 1), generator=g) * 1e-2 + 1e-3
    cfg = choose_config(m, n, k)

    rows = sample_rows(m)
    a_rows = np_(a)[rows].astype(np.float64)
    acc = (a_rows @ w64.T).astype(np.int32)                   # exact: every sum < 2**53

    got = w8a8_mm(a, w.t(), sa.cuda(), sb.cuda(), raw=True)
    assert np.array_equal(np_(got)[rows], acc), f"int32 product differs under {cfg.name}"

    out = w8a8_mm(a, w.t(), sa.cuda(), sb.cuda(), torch.bfloat16, bias.cuda())
    sa_r = sa.numpy()[rows]
    want = to_bits(og.epilogue_f32(acc, sa_r, sb.numpy(), np_(bias)), "bf16")
    assert np.array_equal(bits(out)[rows], want), f"bf16 output differs under {cfg.name}"
    term, ref = og.scaled_ref(acc, sa_r, sb.numpy(), np_(bias))
    assert og.rel_error(np_(out)[rows], term, ref) < 1e-2
