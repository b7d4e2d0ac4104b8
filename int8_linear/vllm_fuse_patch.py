"""Feed Qwen3's int8 linears from the fused quantising kernels.

For int8 W8A8 models vLLM quantises every linear layer's input in its own kernel
(scaled_int8_quant) after the RMSNorm or SiLU-and-mul that produced it.  This patch
removes that step for three of Qwen3's four linears, in the process that builds the
model (VLLM_ENABLE_V1_MULTIPROCESSING=0):

  * vLLM's int8 linear kernels (Triton and CUTLASS) accept a PreQuant input, an
    activation that is already int8 with its per-token scales, and go straight to the
    matmul;
  * Qwen3's decoder layer feeds qkv_proj and gate_up_proj from add_rmsnorm_quant,
    and its MLP feeds down_proj from silu_mul_quant.

o_proj still quantises its own input (attention's output has no kernel of ours in
front of it).  PREQUANT_CALLS counts matmuls that received a PreQuant, so a patch
that never fired shows up as zero.  Same hooks as the reference module
int8_linear/vllm_fuse_patch.py (AshrithaG/int8-linear).
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

import torch

from int8_linear import fused_quant
from int8_linear.fused_quant import add_rmsnorm_quant_op, rmsnorm_quant_op, silu_mul_quant_op

PREQUANT_CALLS = 0


@dataclass
class PreQuant:
    """An int8 activation quantised per token, with the dtype the matmul should output."""
    data: torch.Tensor
    scale: torch.Tensor
    dtype: torch.dtype


def _decoder_forward(self, positions, hidden_states, residual):
    norm = self.input_layernorm
    if residual is None:
        residual = hidden_states
        q, s = rmsnorm_quant_op(hidden_states, norm.weight, norm.variance_epsilon)
    else:
        q, s, residual = add_rmsnorm_quant_op(hidden_states, residual, norm.weight,
                                              norm.variance_epsilon)
    hidden_states = self.self_attn(positions=positions,
                                   hidden_states=PreQuant(q, s, residual.dtype))
    norm = self.post_attention_layernorm
    q, s, residual = add_rmsnorm_quant_op(hidden_states, residual, norm.weight,
                                          norm.variance_epsilon)
    hidden_states = self.mlp(PreQuant(q, s, residual.dtype))
    return hidden_states, residual


def _mlp_forward(self, x):
    gate_up, _ = self.gate_up_proj(x)
    q, s = silu_mul_quant_op(gate_up)
    out, _ = self.down_proj(PreQuant(q, s, gate_up.dtype))
    return out


def _wrap_apply(cls, matmul):
    """Make cls.apply_weights take a PreQuant straight to `matmul`; anything else
    takes the original path."""
    original = cls.apply_weights

    def apply_weights(self, layer, x, bias=None):
        global PREQUANT_CALLS
        if not isinstance(x, PreQuant):
            return original(self, layer, x, bias)
        w_q, w_s, i_s, i_zp, azp_adj = self._get_layer_params(layer)
        if i_s is not None or azp_adj is not None:
            raise NotImplementedError("PreQuant covers symmetric dynamic per-token int8 only")
        PREQUANT_CALLS += 1
        return matmul(x.data, w_q, x.scale, w_s, x.dtype, bias)

    apply_weights._fuse_patched = True
    cls.apply_weights = apply_weights


def use_measured_numerics(path: Path = Path("results/fuse_numerics.json")) -> None:
    """Set the fused kernels' division and SiLU rounding from a numerics study
    ({"best_precise_div": bool, "best_round_silu": bool}) when the file exists."""
    if path.exists():
        num = json.loads(path.read_text())
        fused_quant.PRECISE_DIV = num["best_precise_div"]
        fused_quant.ROUND_SILU = num["best_round_silu"]


def patch_vllm() -> None:
    use_measured_numerics()
    from vllm import _custom_ops as ops
    from vllm.model_executor.kernels.linear.scaled_mm import cutlass
    from vllm.model_executor.kernels.linear.scaled_mm import triton as vllm_triton
    from vllm.model_executor.models import qwen2, qwen3

    if not getattr(vllm_triton.TritonInt8ScaledMMLinearKernel.apply_weights, "_fuse_patched", False):
        # Through the module attribute, so int8_linear.vllm_patch's GEMM swap is honoured.
        _wrap_apply(vllm_triton.TritonInt8ScaledMMLinearKernel,
                    lambda a, w, sa, sb, dt, b: vllm_triton.triton_scaled_mm(
                        a, w, scale_a=sa, scale_b=sb, out_dtype=dt, bias=b))
        _wrap_apply(cutlass.CutlassInt8ScaledMMLinearKernel,
                    lambda a, w, sa, sb, dt, b: ops.cutlass_scaled_mm(
                        a, w, scale_a=sa, scale_b=sb, out_dtype=dt, bias=b))
    qwen3.Qwen3DecoderLayer.forward = _decoder_forward
    qwen2.Qwen2MLP.forward = _mlp_forward
