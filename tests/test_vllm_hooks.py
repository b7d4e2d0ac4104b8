"""The vLLM hooks: int8_linear.vllm_patch and int8_linear.vllm_fuse_patch.

Ports the reference's behaviour specs for them:
  tests/test_vllm_patch.py:20-71   the op equals the kernel; under torch.compile the tile
                                   is chosen from the runtime batch; eager calls skip the
                                   custom op; a declined shape goes to the replaced kernel
                                   and FALLBACKS counts it;
  tests/test_fused_quant.py:100-139  the custom quantiser ops pass opcheck; a PreQuant
                                   goes straight to the matmul (PREQUANT_CALLS counts it)
                                   while a plain tensor takes the original path; static or
                                   asymmetric quantisation is refused.
Plus: a reference-style tiling (Config(16, 64, 64, 4, 1, 1), a Triton tile this library
has no kernel for) reaching scaled_mm falls back instead of failing.

The routing tests need no GPU; the rest are marked gpu.
"""

from __future__ import annotations

import pytest
import torch

from int8_linear import vllm_fuse_patch as vfp
from int8_linear import vllm_patch

EPS = 1e-6
gpu = pytest.mark.gpu


def operands(m, k, n, seed, low=-127, high=128):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randint(low, high, (m, k), dtype=torch.int8, device="cuda", generator=g)
    w = torch.randint(low, high, (n, k), dtype=torch.int8, device="cuda", generator=g)
    sa = torch.rand((m, 1), device="cuda", generator=g) * 1e-2 + 1e-3
    sb = torch.rand((n, 1), device="cuda", generator=g) * 1e-2 + 1e-3
    return a, w.t(), sa, sb


def rand(shape, seed, scale=1.0, dtype=torch.bfloat16):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(shape, generator=g, device="cuda") * scale).to(dtype)


@gpu
def test_op_matches_kernel():
    from int8_linear.kernel import w8a8_mm

    a, w, sa, sb = operands(64, 2048, 4096, 1)
    got = vllm_patch.scaled_mm(a, w, scale_a=sa, scale_b=sb, out_dtype=torch.bfloat16)
    assert torch.equal(got, w8a8_mm(a, w, sa, sb, torch.bfloat16))
    # and through the registered custom op itself
    op = torch.ops.int8_linear.w8a8_mm(a, w, sa, sb, torch.bfloat16, None)
    assert torch.equal(op, got)


@gpu
def test_compiled_op_configures_from_runtime_batch():
    """If the tile were chosen at trace time, both batch sizes would share it."""

    def layer(a, w, sa, sb):
        return vllm_patch.scaled_mm(a, w, scale_a=sa, scale_b=sb, out_dtype=torch.bfloat16)

    compiled = torch.compile(layer, fullgraph=True, dynamic=True)
    vllm_patch.CONFIGS.clear()
    outs = {}
    for m in (3, 700):
        ops = operands(m, 2048, 2048, m)
        outs[m] = (compiled(*ops), layer(*ops))
    chosen = {m: name for (m, _, _), name in vllm_patch.CONFIGS.items()}
    assert chosen[3] != chosen[700], chosen
    for m, (got, want) in outs.items():
        assert torch.equal(got, want)


@gpu
def test_eager_calls_skip_the_custom_op(monkeypatch):
    from int8_linear.kernel import w8a8_mm

    def custom_op(*args):
        raise AssertionError("an eager call went through the custom op")

    monkeypatch.setattr(vllm_patch, "w8a8_mm_op", custom_op)
    a, w, sa, sb = operands(16, 2048, 2048, 4)
    got = vllm_patch.scaled_mm(a, w, scale_a=sa, scale_b=sb, out_dtype=torch.bfloat16)
    assert torch.equal(got, w8a8_mm(a, w, sa, sb, torch.bfloat16))


@gpu
def test_declined_shapes_go_to_the_replaced_kernel(monkeypatch):
    seen = []

    def replaced(a, w, sa, sb, out_dtype, bias):
        seen.append(tuple(a.shape))
        return torch.zeros((a.shape[0], w.shape[1]), dtype=out_dtype, device=a.device)

    monkeypatch.setattr(vllm_patch, "_vllm_triton_scaled_mm", replaced)
    before = vllm_patch.FALLBACKS
    a, w, sa, sb = operands(4, 100, 64, 2)  # K=100: no 16-byte rows for TMA
    out = vllm_patch.scaled_mm(a, w, scale_a=sa, scale_b=sb, out_dtype=torch.bfloat16)
    assert seen == [(4, 100)] and vllm_patch.FALLBACKS == before + 1
    assert tuple(out.shape) == (4, 64)


@gpu
def test_reference_style_tiling_falls_back(monkeypatch):
    """A tile from the reference's Triton table (bm, bn, bk, warps, stages, group_m) has no
    B200 kernel: w8a8_mm raises NotSupported for it, and scaled_mm hands the call to the
    replaced vLLM kernel instead of failing."""
    from int8_linear import Config, NotSupported, w8a8_mm

    ref_tile = Config(16, 64, 64, 4, 1, 1)
    a, w, sa, sb = operands(16, 2048, 2048, 9)
    with pytest.raises(NotSupported):
        w8a8_mm(a, w, sa, sb, torch.bfloat16, config=ref_tile)
    seen = []

    def replaced(a_, w_, sa_, sb_, out_dtype, bias):
        seen.append(tuple(a_.shape))
        return torch.full((a_.shape[0], w_.shape[1]), 7.0, dtype=out_dtype, device=a_.device)

    monkeypatch.setattr(vllm_patch, "_vllm_triton_scaled_mm", replaced)
    monkeypatch.setattr(vllm_patch, "choose_config", lambda m, n, k: ref_tile)
    before = vllm_patch.FALLBACKS
    out = vllm_patch.scaled_mm(a, w, scale_a=sa, scale_b=sb, out_dtype=torch.bfloat16)
    assert seen == [(16, 2048)] and vllm_patch.FALLBACKS == before + 1
    assert bool((out == 7.0).all())


@gpu
def test_custom_ops_opcheck():
    from int8_linear import fused_quant as fq

    x, r = rand((9, 2048), 1), rand((9, 2048), 2)
    w = rand((2048,), 3) + 1.0
    torch.library.opcheck(fq.rmsnorm_quant_op, (x, w, EPS))
    torch.library.opcheck(fq.add_rmsnorm_quant_op, (x, r, w, EPS))
    torch.library.opcheck(fq.silu_mul_quant_op, (rand((9, 2 * 6144), 4),))
    torch.library.opcheck(fq.per_token_quant_op, (x,))
    a, w8, sa, sb = operands(9, 2048, 1024, 5)
    torch.library.opcheck(vllm_patch.w8a8_mm_op, (a, w8, sa, sb, torch.bfloat16, None))


def test_prequant_routing():
    """A PreQuant goes straight to the matmul; a plain tensor takes the original path."""
    calls = []

    class Kernel:
        def _get_layer_params(self, layer):
            return "w_q", "w_s", None, None, None

        def apply_weights(self, layer, x, bias=None):
            calls.append("original")
            return "orig"

    vfp._wrap_apply(Kernel, lambda a, w, sa, sb, dt, b: calls.append((a, w, sa, sb, dt, b)) or "fast")
    before = vfp.PREQUANT_CALLS
    k = Kernel()
    assert k.apply_weights(None, vfp.PreQuant("q", "s", torch.bfloat16), "b") == "fast"
    assert calls[-1] == ("q", "w_q", "s", "w_s", torch.bfloat16, "b")
    assert vfp.PREQUANT_CALLS == before + 1
    assert k.apply_weights(None, torch.zeros(1)) == "orig"
    assert calls[-1] == "original" and vfp.PREQUANT_CALLS == before + 1


@pytest.mark.parametrize("params", [("w_q", "w_s", "static_scale", None, None),
                                    ("w_q", "w_s", None, "zero_point", "azp_adj")])
def test_prequant_rejects_static_or_asymmetric(params):
    class Kernel:
        def _get_layer_params(self, layer):
            return params

        def apply_weights(self, layer, x, bias=None):
            return "orig"

    vfp._wrap_apply(Kernel, lambda *a: "fast")
    with pytest.raises(NotImplementedError):
        Kernel().apply_weights(None, vfp.PreQuant("q", "s", torch.bfloat16))
