"""The stand-in decoder step against the oracle, op by op.

The reference times its fused path on a 28-layer stand-in (bench/fuse_quant.py:226-240,
Stack.fused):

    add_rmsnorm_quant -> qkv_proj -> [:, :2048] per-token quant -> o_proj
    -> add_rmsnorm_quant (residual) -> gate_up_proj -> silu_mul_quant -> down_proj

with the next layer's add_rmsnorm_quant taking down_proj's output and the residual.
Here every op of a 3-layer StandinDecoder step is recorded and checked on its own GPU
inputs: each GEMM's bf16 output bit for bit against the fp32 epilogue of the exact int32
product, each quantiser within the reference's tolerance (tests/test_fused_quant.py:54-61)
with the residual bit-exact, the plain per-token quantiser bit-exact; and the recorded
ops are checked to chain exactly as the reference composes them (each op's input is the
output the composition says it is).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from int8_linear.standin import EPS, HIDDEN, StandinDecoder
from oracle import gemm as og
from oracle import quant as oq
from oracle.numerics import to_bits
from tests.gpu_util import bits, np_

pytestmark = pytest.mark.gpu

ORDER = ["qkv_proj", "quant", "o_proj", "post_norm", "gate_up_proj", "silu_mul_quant", "down_proj"]


def same(a: torch.Tensor, b: torch.Tensor) -> bool:
    """The same tensor (storage, offset, shape and strides), not just equal values."""
    return (a.data_ptr() == b.data_ptr() and a.shape == b.shape and a.stride() == b.stride()
            and a.dtype == b.dtype)


def check_gemm(ins, out):
    q, s, lin = ins
    w = lin.w_t.t()
    acc = og.exact(np_(q), np_(w))
    want = to_bits(og.epilogue_f32(acc, np_(s), np_(lin.scale)), "bf16")
    assert np.array_equal(bits(out), want)


def check_norm(ins, outs):
    x, r, w = ins
    q, s, rout = outs
    q0, s0, r0 = oq.ref_norm(np_(x), np_(r) if r is not None else None, np_(w), EPS,
                             quantiser=oq.quant_ieee, kernel_order=True)
    d = oq.compare_int8(np_(q), np_(s), q0, s0)
    assert d.ok(), d
    if r is not None:
        assert np.array_equal(bits(rout), to_bits(r0, "bf16"))


@pytest.mark.parametrize("m", [1, 16, 128])
@pytest.mark.parametrize("gamma", ["ones", "config3"])
def test_every_op_of_the_step_matches_the_oracle(m, gamma):
    g = torch.Generator().manual_seed(5)
    w = (torch.ones(HIDDEN) if gamma == "ones" else 1.0 + 0.1 * torch.randn(HIDDEN, generator=g))
    dec = StandinDecoder(m, layers=3, norm_weight=w.to(torch.bfloat16).cuda(), fuse=False)
    rec: list = []
    out = dec.step(record=rec)
    torch.cuda.synchronize()

    # the composition: one input norm, then per layer the seven ops in the reference's
    # order, the norm of the next layer between them
    names = [(i, n) for i, n, _, _ in rec]
    want = [(-1, "norm")]
    for i in range(3):
        want += ([(i, "norm")] if i else []) + [(i, n) for n in ORDER]
    assert names == want

    prev_out = {}
    res = dec.x
    for i, name, ins, outs in rec:
        if name == "norm":
            x, r, _ = ins
            if i == -1:
                assert same(x, dec.x) and r is None
            else:
                assert same(x, prev_out["down_proj"]) and same(r, res)
                res = outs[2]
            check_norm(ins, outs)
        elif name == "post_norm":
            x, r, _ = ins
            assert same(x, prev_out["o_proj"]) and same(r, res)
            res = outs[2]
            check_norm(ins, outs)
        elif name == "quant":
            (x,) = ins
            qkv = prev_out["qkv_proj"]
            assert x.data_ptr() == qkv.data_ptr() and x.shape == (m, HIDDEN)   # qkv[:, :2048]
            q0, s0 = oq.quant_ieee(np_(x))
            assert np.array_equal(np_(outs[0]), q0) and np.array_equal(np_(outs[1]), s0)
        elif name == "silu_mul_quant":
            (gu,) = ins
            assert same(gu, prev_out["gate_up_proj"])
            q0, s0 = oq.ref_silu(np_(gu), False, quantiser=oq.quant_ieee)
            d = oq.compare_int8(np_(outs[0]), np_(outs[1]), q0, s0)
            assert d.ok(), d
        else:
            q, s, lin = ins
            feeder = {"qkv_proj": "norm", "o_proj": "quant", "gate_up_proj": "post_norm",
                      "down_proj": "silu_mul_quant"}[name]
            src = prev_out[feeder]
            assert same(q, src[0]) and same(s, src[1])
            assert lin is dec.layers[i][name]
            check_gemm(ins, outs)
        prev_out[name] = outs
    assert same(out, prev_out["down_proj"])


@pytest.mark.parametrize("m", [1, 2, 3, 4, 8, 16])
def test_fused_step_equals_the_step_of_separate_ops(m):
    """With the quantisers in the GEMM prologues (CUDA-core tiles) the step gives the
    same bits as the step of separate quantiser and GEMM launches, eagerly and replayed
    from a CUDA graph; and the fused ops really ran as fused kernels where they can."""
    g = torch.Generator().manual_seed(6)
    w = (1.0 + 0.1 * torch.randn(HIDDEN, generator=g)).to(torch.bfloat16).cuda()
    dec = StandinDecoder(m, layers=3, norm_weight=w, fuse=False)
    want = dec.step().clone()
    assert dec.launches_per_step == 1 + 7 * 3 + 2
    dec.fuse = {"qkv_proj", "o_proj", "gate_up_proj", "down_proj"}
    assert torch.equal(dec.step(), want)
    dec.capture().replay()
    torch.cuda.synchronize()
    assert torch.equal(dec.out, want)
    if m <= 2:   # every quantiser fused: 4 launches per layer
        assert dec.launches_per_step == 4 * 3
    dec.fuse = True    # the measured per-batch choice
    assert torch.equal(dec.step(), want)
