"""The activation quantiser fused into the kernel before it, on B200 (sm_100a).

A W8A8 int8 layer quantises its input per token right before the matmul.  These
kernels fold that quantiser into the op that produces the input, so the activation
is written once, as int8, instead of being written in bf16 and read back:

    add_rmsnorm_quant(x, residual, w, eps) -> (x_q, scale, residual_out)
    rmsnorm_quant(x, w, eps)               -> (x_q, scale)
    silu_mul_quant(gate_up)                -> (x_q, scale)
    per_token_quant(x)                     -> (x_q, scale)   (no op before it)

Same Python API and arithmetic as the reference module int8_linear/fused_quant.py
(AshrithaG/int8-linear): the residual add and the norm in fp32, the normalised value
rounded to the weight dtype before and to the activation dtype after the weight
multiply, then the dynamic per-token quantiser

    scale = absmax / 127,   x_q = round_half_even(x * (127 / absmax)), saturated

PRECISE_DIV picks IEEE division for those two divides or the approximate full-range
one; ROUND_SILU rounds silu(gate) to the activation dtype before the multiply.  The
kernels are the hand-written sm_100a CUDA in csrc/quant.cu behind the C ABI; each is
also a torch custom op, so torch.compile treats it as one opaque kernel.
"""

from __future__ import annotations

import torch

from int8_linear import _native
from int8_linear._native import NotSupported
from int8_linear.kernel import current_stream

_ACT = {torch.bfloat16: _native.BF16, torch.float16: _native.F16}
_WEIGHT = {torch.bfloat16: _native.BF16, torch.float16: _native.F16, torch.float32: _native.F32}


def _act_code(t: torch.Tensor) -> int:
    if t.dtype not in _ACT:
        raise NotSupported(f"activations must be bfloat16 or float16, got {t.dtype}")
    if not t.is_cuda:
        raise ValueError(f"the fused quantisers run on a CUDA device, got {t.device}")
    return _ACT[t.dtype]


def _stream(t: torch.Tensor) -> int:
    return current_stream(t.get_device())


def add_rmsnorm_quant(x: torch.Tensor, residual: torch.Tensor | None, weight: torch.Tensor,
                      eps: float, precise_div: bool = True):
    """(x_q int8 [M, K], scale fp32 [M, 1], residual_out [M, K] or None)."""
    assert x.is_contiguous() and x.dim() == 2
    M, K = x.shape
    act = _act_code(x)
    if weight.dtype not in _WEIGHT or weight.numel() != K:
        raise ValueError(f"weight must hold {K} bf16/fp16/fp32 values, got {weight.dtype} "
                         f"{tuple(weight.shape)}")
    q = torch.empty((M, K), dtype=torch.int8, device=x.device)
    s = torch.empty((M, 1), dtype=torch.float32, device=x.device)
    rout = torch.empty_like(x) if residual is not None else None
    if residual is not None:
        assert residual.shape == x.shape and residual.dtype == x.dtype and residual.stride(1) == 1
    if M:
        w = weight.contiguous()
        _native.check(_native.load().i8l_add_rmsnorm_quant(
            x.data_ptr(), x.stride(0),
            residual.data_ptr() if residual is not None else None,
            residual.stride(0) if residual is not None else 0,
            w.data_ptr(), act, _WEIGHT[w.dtype], q.data_ptr(), q.stride(0), s.data_ptr(),
            rout.data_ptr() if rout is not None else None, rout.stride(0) if rout is not None else 0,
            M, K, float(eps), int(bool(precise_div)), _stream(x)))
    return q, s, rout


def silu_mul_quant(gate_up: torch.Tensor, precise_div: bool = True, round_silu: bool = False,
                   absmax: torch.Tensor | None = None):
    """silu(gate) * up, quantised: (x_q int8 [M, I], scale fp32 [M, 1]).  `absmax` ([M]
    float32, e.g. the MAX over the GPUs sharing each row) replaces each row's own
    max|y|, as for a row split across GPUs (see silu_mul_absmax)."""
    assert gate_up.is_contiguous() and gate_up.dim() == 2
    M, I2 = gate_up.shape
    I = I2 // 2
    act = _act_code(gate_up)
    q = torch.empty((M, I), dtype=torch.int8, device=gate_up.device)
    s = torch.empty((M, 1), dtype=torch.float32, device=gate_up.device)
    if M and I:
        amax = _absmax_arg(absmax, M)
        _native.check(_native.load().i8l_silu_mul_quant_ex(
            gate_up.data_ptr(), gate_up.stride(0), act, q.data_ptr(), q.stride(0), s.data_ptr(),
            M, I, int(bool(precise_div)), int(bool(round_silu)),
            amax.data_ptr() if amax is not None else None, None, _stream(gate_up)))
    return q, s


def silu_mul_absmax(gate_up: torch.Tensor, round_silu: bool = False) -> torch.Tensor:
    """max over each row of |silu(gate) * up| (float32 [M]), the first half of a
    SiLU-and-mul quantisation whose row is split across GPUs."""
    assert gate_up.is_contiguous() and gate_up.dim() == 2
    M, I = gate_up.shape[0], gate_up.shape[1] // 2
    act = _act_code(gate_up)
    out = torch.empty((M,), dtype=torch.float32, device=gate_up.device)
    if M and I:
        _native.check(_native.load().i8l_silu_mul_quant_ex(
            gate_up.data_ptr(), gate_up.stride(0), act, None, 0, None, M, I, 1,
            int(bool(round_silu)), None, out.data_ptr(), _stream(gate_up)))
    return out


def _absmax_arg(absmax: torch.Tensor | None, m: int) -> torch.Tensor | None:
    if absmax is None:
        return None
    absmax = absmax.reshape(-1).contiguous()
    if absmax.dtype != torch.float32 or absmax.numel() != m:
        raise ValueError(f"absmax must hold {m} float32 values, got {absmax.dtype} {tuple(absmax.shape)}")
    return absmax


def per_token_quant(x: torch.Tensor, precise_div: bool = True, absmax: torch.Tensor | None = None):
    """Dynamic symmetric per-token int8 quantisation of a 2-D activation whose rows
    are contiguous (a column slice of a wider matrix is fine, no copy is made):
    (x_q int8 [M, K], scale fp32 [M, 1]).  This is the step the reference leaves to
    vLLM's scaled_int8_quant before o_proj (bench/fuse_quant.py:234).  `absmax`
    ([M] float32) replaces each row's own max|x|, for rows split across GPUs."""
    assert x.dim() == 2 and x.stride(1) == 1
    M, K = x.shape
    act = _act_code(x)
    q = torch.empty((M, K), dtype=torch.int8, device=x.device)
    s = torch.empty((M, 1), dtype=torch.float32, device=x.device)
    if M and K:
        amax = _absmax_arg(absmax, M)
        _native.check(_native.load().i8l_quant_rows_ex(
            x.data_ptr(), x.stride(0), act, q.data_ptr(), q.stride(0), s.data_ptr(), M, K,
            int(bool(precise_div)), amax.data_ptr() if amax is not None else None, None, _stream(x)))
    return q, s


def row_absmax(x: torch.Tensor) -> torch.Tensor:
    """max over each row of |x| (float32 [M]) for a bf16/fp16 matrix with contiguous rows."""
    assert x.dim() == 2 and x.stride(1) == 1
    M, K = x.shape
    act = _act_code(x)
    out = torch.empty((M,), dtype=torch.float32, device=x.device)
    if M and K:
        _native.check(_native.load().i8l_quant_rows_ex(
            x.data_ptr(), x.stride(0), act, None, 0, None, M, K, 1, None, out.data_ptr(), _stream(x)))
    return out


# Numerics the custom ops use.  The reference measures which choice matches vLLM and
# its served path sets both to True (results/fuse_numerics.json there).
PRECISE_DIV = True
ROUND_SILU = False


@torch.library.custom_op("int8_linear::rmsnorm_quant", mutates_args=())
def rmsnorm_quant_op(x: torch.Tensor, weight: torch.Tensor, eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    q, s, _ = add_rmsnorm_quant(x.contiguous(), None, weight, eps, PRECISE_DIV)
    return q, s


@rmsnorm_quant_op.register_fake
def _(x, weight, eps):
    return (x.new_empty(x.shape, dtype=torch.int8),
            x.new_empty((x.shape[0], 1), dtype=torch.float32))


@torch.library.custom_op("int8_linear::add_rmsnorm_quant", mutates_args=())
def add_rmsnorm_quant_op(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                         eps: float) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    return add_rmsnorm_quant(x.contiguous(), residual.contiguous(), weight, eps, PRECISE_DIV)


@add_rmsnorm_quant_op.register_fake
def _(x, residual, weight, eps):
    return (x.new_empty(x.shape, dtype=torch.int8),
            x.new_empty((x.shape[0], 1), dtype=torch.float32),
            torch.empty_like(x))


@torch.library.custom_op("int8_linear::silu_mul_quant", mutates_args=())
def silu_mul_quant_op(gate_up: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    return silu_mul_quant(gate_up.contiguous(), PRECISE_DIV, ROUND_SILU)


@silu_mul_quant_op.register_fake
def _(gate_up):
    return (gate_up.new_empty((gate_up.shape[0], gate_up.shape[1] // 2), dtype=torch.int8),
            gate_up.new_empty((gate_up.shape[0], 1), dtype=torch.float32))


@torch.library.custom_op("int8_linear::per_token_quant", mutates_args=())
def per_token_quant_op(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    return per_token_quant(x.contiguous(), PRECISE_DIV)


@per_token_quant_op.register_fake
def _(x):
    return (x.new_empty(x.shape, dtype=torch.int8),
            x.new_empty((x.shape[0], 1), dtype=torch.float32))
