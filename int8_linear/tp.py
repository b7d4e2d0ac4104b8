"""Tensor-parallel W8A8 linears across the GPUs of one node (torch.distributed).

The reference is single-GPU; this is the B200 extension for layers too large for one
GPU or decode steps split across several.  Megatron-style sharding:

* ColumnParallelW8A8 (qkv, gate_up): each rank holds output rows W[N/g, K] with their
  scales and bias; the activation is replicated; each rank's output columns are
  independent (an optional NCCL all-gather assembles [M, N]).  No data-path collective.
* RowParallelW8A8 (o_proj, down): each rank holds W[:, K/g] and the int8 slice of the
  activation; the int32 partial products are summed over the ranks (all-reduce SUM on
  int32: exact and order-free) and dequantised once, so the output equals the one-GPU
  GEMM bit for bit.
* The activation of a row-parallel layer is split along its row, so its per-token scale
  needs the row's global max|x|: each rank computes its local absmax, an all-reduce MAX
  gives the global one, and every rank quantises its slice with it (sharded_*_quant),
  exactly as one GPU would quantise the whole row.

All tensor arithmetic goes through an `ops` object: CudaOps (this library's sm_100a
kernels) by default; tests substitute a CPU implementation to check the sharding and
collective logic with gloo ranks.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


class CudaOps:
    """The sm_100a kernels of this library."""

    def mm_raw(self, a_q, w):
        from int8_linear.kernel import w8a8_mm
        one = torch.ones(1, device=a_q.device)
        return w8a8_mm(a_q, w.t(), one, one, raw=True)

    def mm(self, a_q, a_s, w, w_s, out_dtype, bias):
        from int8_linear.kernel import w8a8_mm
        return w8a8_mm(a_q, w.t(), a_s, w_s, out_dtype, bias)

    def dequant(self, acc, a_s, w_s, out_dtype, bias):
        from int8_linear.kernel import dequant_i32
        return dequant_i32(acc, a_s, w_s, out_dtype, bias)

    def absmax(self, x):
        from int8_linear.fused_quant import row_absmax
        return row_absmax(x)

    def quant(self, x, absmax=None):
        from int8_linear.fused_quant import per_token_quant
        return per_token_quant(x, absmax=absmax)

    def silu_absmax(self, gate_up, round_silu):
        from int8_linear.fused_quant import silu_mul_absmax
        return silu_mul_absmax(gate_up, round_silu)

    def silu_quant(self, gate_up, round_silu, absmax=None):
        from int8_linear.fused_quant import silu_mul_quant
        return silu_mul_quant(gate_up, True, round_silu, absmax=absmax)


def shard_rows_of(x: torch.Tensor, rank: int, world: int, parts: tuple[int, ...] | None = None):
    """Rank's share of the first dimension.  `parts` splits a merged weight (e.g. q, k, v
    or gate, up) into segments that are sharded separately, Megatron-style."""
    parts = parts or (x.shape[0],)
    assert sum(parts) == x.shape[0]
    out, start = [], 0
    for p in parts:
        assert p % world == 0, f"segment of {p} rows does not split over {world} ranks"
        step = p // world
        out.append(x[start + rank * step: start + (rank + 1) * step])
        start += p
    return torch.cat(out, dim=0).contiguous()


def shard_cols_of(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Rank's share of the last dimension (the K of a row-parallel weight)."""
    k = x.shape[-1]
    assert k % world == 0, f"K={k} does not split over {world} ranks"
    step = k // world
    return x[..., rank * step:(rank + 1) * step].contiguous()


@dataclass
class ColumnParallelW8A8:
    """Output-column shard of an int8 linear: w [N/g, K] int8, w_s [N/g, 1] fp32."""
    w: torch.Tensor
    w_s: torch.Tensor
    bias: torch.Tensor | None = None
    group: dist.ProcessGroup | None = None
    ops: object = None

    def __post_init__(self):
        self.ops = self.ops or CudaOps()

    def __call__(self, a_q, a_s, out_dtype=torch.bfloat16, gather: bool = False):
        local = self.ops.mm(a_q, a_s, self.w, self.w_s, out_dtype, self.bias)
        if not gather:
            return local
        world = dist.get_world_size(self.group)
        m, n = local.shape
        full = torch.empty((world * m, n), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(full, local.contiguous(), group=self.group)
        return full.view(world, m, n).permute(1, 0, 2).reshape(m, world * n)


@dataclass
class RowParallelW8A8:
    """Input-row shard of an int8 linear: w [N, K/g] int8, w_s [N, 1] fp32 (whole),
    bias [N] (whole, added once after the reduction)."""
    w: torch.Tensor
    w_s: torch.Tensor
    bias: torch.Tensor | None = None
    group: dist.ProcessGroup | None = None
    ops: object = None

    def __post_init__(self):
        self.ops = self.ops or CudaOps()

    def __call__(self, a_q_shard, a_s, out_dtype=torch.bfloat16):
        """a_q_shard: this rank's int8 columns [M, K/g]; a_s: the GLOBAL per-token scale."""
        acc = self.ops.mm_raw(a_q_shard, self.w)
        dist.all_reduce(acc, op=dist.ReduceOp.SUM, group=self.group)
        return self.ops.dequant(acc, a_s, self.w_s, out_dtype, self.bias)


def sharded_per_token_quant(x_shard, group=None, ops=None):
    """Per-token int8 of a row split over the ranks (x_shard [M, K/g]), with the scale of
    the whole row: (q_shard, scale [M, 1]) identical to one GPU's on the full row."""
    ops = ops or CudaOps()
    amax = ops.absmax(x_shard)
    dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=group)
    return ops.quant(x_shard, absmax=amax)


def sharded_silu_mul_quant(gate_up_shard, round_silu: bool = False, group=None, ops=None):
    """SiLU-and-mul + per-token int8 of gate||up columns split over the ranks
    (gate_up_shard = [gate_r | up_r], [M, 2 I/g]), with the whole row's scale."""
    ops = ops or CudaOps()
    amax = ops.silu_absmax(gate_up_shard, round_silu)
    dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=group)
    return ops.silu_quant(gate_up_shard, round_silu, absmax=amax)
