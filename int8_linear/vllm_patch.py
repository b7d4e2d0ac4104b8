"""Put this library's GEMM into vLLM's Triton int8 linear path.

vLLM's TritonInt8ScaledMMLinearKernel.apply_weights calls the module-level name
``triton_scaled_mm(input, weight, scale_a=..., scale_b=..., out_dtype=..., bias=...)``
of vllm.model_executor.kernels.linear.scaled_mm.triton.  patch_vllm() rebinds that
one name to scaled_mm below, so only the matmul changes: weight loading, vLLM's
activation quantiser and its dispatch stay as they are.  Same hook as the reference
module int8_linear/vllm_patch.py (AshrithaG/int8-linear).

While torch.compile traces, scaled_mm goes through the custom op
int8_linear::w8a8_mm, so the tile is chosen from the real batch size at run time
instead of being frozen at trace time.  Eager calls skip the op and launch directly
(the op's dispatch costs host time on every call).  A shape the kernel declines
goes to the replaced vLLM function and FALLBACKS counts it.

vLLM must build the model in this process (VLLM_ENABLE_V1_MULTIPROCESSING=0) for
the patch to reach it.
"""

from typing import Optional

import torch

from int8_linear.kernel import NotSupported, choose_config, tuned_config, w8a8_mm

# Calls that reached the kernel, calls it declined, and the tile each (M, K, N)
# used.  Under CUDA graphs Python runs only at warm-up and capture, so a patched
# model that never reached the kernel shows CALLS == 0.
CALLS = 0
FALLBACKS = 0
CONFIGS: dict[tuple[int, int, int], str] = {}
_vllm_triton_scaled_mm = None


def _run(a_q: torch.Tensor, b_q: torch.Tensor, scale_a: torch.Tensor, scale_b: torch.Tensor,
         out_dtype: torch.dtype, bias: Optional[torch.Tensor]) -> torch.Tensor:
    global CALLS, FALLBACKS
    m, k = a_q.shape
    n = b_q.shape[1]
    cfg = choose_config(m, n, k)
    CALLS += 1
    CONFIGS.setdefault((m, k, n), cfg.name)
    try:
        return w8a8_mm(a_q, b_q, scale_a, scale_b, out_dtype, bias, config=cfg)
    except NotSupported:
        if _vllm_triton_scaled_mm is None:
            raise
        FALLBACKS += 1
        return _vllm_triton_scaled_mm(a_q, b_q, scale_a, scale_b, out_dtype, bias)


@torch.library.custom_op("int8_linear::w8a8_mm", mutates_args=())
def w8a8_mm_op(a_q: torch.Tensor, b_q: torch.Tensor, scale_a: torch.Tensor,
               scale_b: torch.Tensor, out_dtype: torch.dtype,
               bias: Optional[torch.Tensor]) -> torch.Tensor:
    return _run(a_q, b_q, scale_a, scale_b, out_dtype, bias)


@w8a8_mm_op.register_fake
def _(a_q, b_q, scale_a, scale_b, out_dtype, bias):
    return a_q.new_empty((a_q.shape[0], b_q.shape[1]), dtype=out_dtype)


def scaled_mm(input: torch.Tensor, weight: torch.Tensor, scale_a: torch.Tensor,
              scale_b: torch.Tensor, out_dtype: torch.dtype,
              bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Drop-in for vLLM's triton_scaled_mm (same signature): the custom op while
    torch.compile traces, the kernel directly otherwise."""
    if torch.compiler.is_compiling():
        return w8a8_mm_op(input, weight, scale_a, scale_b, out_dtype, bias)
    return _run(input, weight, scale_a, scale_b, out_dtype, bias)


def patch_vllm() -> None:
    """Rebind vLLM's triton_scaled_mm to scaled_mm (idempotent)."""
    global _vllm_triton_scaled_mm
    import vllm.model_executor.kernels.linear.scaled_mm.triton as vllm_triton_kernel

    if vllm_triton_kernel.triton_scaled_mm is not scaled_mm:
        _vllm_triton_scaled_mm = vllm_triton_kernel.triton_scaled_mm
    # Read the tile table now, so no file is opened inside a traced or captured region.
    tuned_config(1, 1, 1)
    vllm_triton_kernel.triton_scaled_mm = scaled_mm
