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

With a PeerComm (NVLink exchange buffers mapped on every GPU of the group) the
collectives run inside this library's own kernels instead of NCCL, fused with the
work around them: the row-parallel int32 sum with the dequant (and, in the stand-in,
with the residual add + RMSNorm + quantiser that follow), the global-absmax MAX with
the split-row quantisers.  Same results bit for bit; one kernel instead of a
collective plus one to three kernels.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist

from int8_linear import _native


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


class PeerComm:
    """One NVLink exchange buffer per GPU of `group`, mapped by every other GPU through a
    CUDA IPC handle (exchanged with all_gather_object).  `slot_bytes` bounds what one GPU
    sends per call (8 bytes per int32 value of a row-parallel all-reduce, as each travels
    with the call's epoch; 16 bytes per row for an absmax), `max_rows` the rows
    per call.  Calls that exceed them raise NotSupported (the callers fall back to NCCL).
    `two_shot_rows`: batches from which the row-parallel sums run as reduce-scatter +
    all-gather instead of one all-to-all (0: the library's choice, 16 rows from 4 GPUs;
    negative: never).  Every GPU of the group must make the same calls in the same order."""

    def __init__(self, group=None, slot_bytes: int = 8 << 20, max_rows: int = 4096,
                 timeout_ns: int = 0, device: torch.device | None = None, two_shot_rows: int = 0):
        lib = _native.load()
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if self.world > _native.MAX_RANKS:
            raise _native.NotSupported(f"peer exchange takes at most {_native.MAX_RANKS} GPUs")
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self._own = ctypes.c_void_p()
        self._opened: list[int] = []
        with torch.cuda.device(self.device):
            nbytes = lib.i8l_peer_buffer_bytes(slot_bytes, self.world)
            if nbytes == 0:
                raise ValueError(f"slot_bytes={slot_bytes} must be a positive multiple of 16")
            handle = (ctypes.c_uint8 * _native.PEER_HANDLE_BYTES)()
            _native.check(lib.i8l_peer_alloc(nbytes, ctypes.byref(self._own), handle))
            handles: list = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
            bases = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    bases.append(self._own.value)
                    continue
                p = ctypes.c_void_p()
                buf = (ctypes.c_uint8 * _native.PEER_HANDLE_BYTES).from_buffer_copy(h)
                _native.check(lib.i8l_peer_open(buf, ctypes.byref(p)))
                self._opened.append(p.value)
                bases.append(p.value)
            self.epochs = torch.zeros(max_rows, dtype=torch.int32, device=self.device)
        self.desc = _native.I8LPeerComm()
        for r, b in enumerate(bases):
            self.desc.bases[r] = b
        self.desc.epochs = self.epochs.data_ptr()
        self.desc.rank, self.desc.world = self.rank, self.world
        self.desc.slot_bytes, self.desc.max_rows = slot_bytes, max_rows
        self.desc.timeout_ns = timeout_ns
        self.desc.two_shot_rows = two_shot_rows
        self.slot_bytes, self.max_rows = slot_bytes, max_rows
        dist.barrier(group=group)   # every buffer is mapped before any GPU signals into it

    def close(self) -> None:
        """Unmap the peers' buffers and free this GPU's (after every GPU is done)."""
        if self._own.value is None:
            return
        lib = _native.load()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self._opened:
                _native.check(lib.i8l_peer_close(ctypes.c_void_p(p)))
            self._opened = []
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            _native.check(lib.i8l_peer_free(self._own))
        self._own = ctypes.c_void_p()

    def fits(self, rows: int, row_bytes: int) -> bool:
        return rows <= self.max_rows and rows * row_bytes <= self.slot_bytes


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


_ACT = {torch.bfloat16: _native.BF16, torch.float16: _native.F16}
_ANY = {torch.bfloat16: _native.BF16, torch.float16: _native.F16, torch.float32: _native.F32}


def peer_allreduce_dequant(comm: PeerComm, acc: torch.Tensor, a_s: torch.Tensor, w_s: torch.Tensor,
                           out_dtype=torch.bfloat16, bias: torch.Tensor | None = None) -> torch.Tensor:
    """Sum of the int32 partials over the GPUs, dequantised like the GEMM epilogue."""
    m, n = acc.shape
    out = torch.empty((m, n), dtype=out_dtype, device=acc.device)
    if m and n:
        _native.check(_native.load().i8l_tp_allreduce_dequant(
            ctypes.byref(comm.desc), acc.data_ptr(), acc.stride(0), a_s.data_ptr(), int(a_s.numel() > 1),
            w_s.data_ptr(), int(w_s.numel() > 1), bias.data_ptr() if bias is not None else None,
            _ANY[bias.dtype] if bias is not None else 0, out.data_ptr(), _ANY[out_dtype], out.stride(0),
            m, n, _stream(acc)))
    return out


def peer_allreduce_add_rmsnorm_quant(comm: PeerComm, acc, a_s, w_s, bias, residual, weight, eps,
                                     precise_div: bool = True, act_dtype=torch.bfloat16,
                                     h_out: torch.Tensor | None = None):
    """The row-parallel layer's sum + dequant to `act_dtype` (h), then
    add_rmsnorm_quant(h, residual, weight, eps) in the same kernel: (q, scale, residual_out)."""
    m, n = acc.shape
    q = torch.empty((m, n), dtype=torch.int8, device=acc.device)
    s = torch.empty((m, 1), dtype=torch.float32, device=acc.device)
    rout = torch.empty((m, n), dtype=act_dtype, device=acc.device) if residual is not None else None
    if m:
        w = weight.contiguous()
        _native.check(_native.load().i8l_tp_allreduce_add_rmsnorm_quant(
            ctypes.byref(comm.desc), acc.data_ptr(), acc.stride(0), a_s.data_ptr(), int(a_s.numel() > 1),
            w_s.data_ptr(), int(w_s.numel() > 1), bias.data_ptr() if bias is not None else None,
            _ANY[bias.dtype] if bias is not None else 0,
            residual.data_ptr() if residual is not None else None,
            residual.stride(0) if residual is not None else 0, w.data_ptr(), _ACT[act_dtype], _ANY[w.dtype],
            q.data_ptr(), q.stride(0), s.data_ptr(), rout.data_ptr() if rout is not None else None,
            rout.stride(0) if rout is not None else 0, h_out.data_ptr() if h_out is not None else None,
            h_out.stride(0) if h_out is not None else 0, m, n, float(eps), int(bool(precise_div)),
            _stream(acc)))
    return q, s, rout


def peer_quant_rows(comm: PeerComm, x: torch.Tensor, precise_div: bool = True):
    """Per-token int8 of this GPU's slice of rows split over the GPUs (global absmax)."""
    assert x.dim() == 2 and x.stride(1) == 1
    m, k = x.shape
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    s = torch.empty((m, 1), dtype=torch.float32, device=x.device)
    if m and k:
        _native.check(_native.load().i8l_tp_quant_rows(
            ctypes.byref(comm.desc), x.data_ptr(), x.stride(0), _ACT[x.dtype], q.data_ptr(), q.stride(0),
            s.data_ptr(), m, k, int(bool(precise_div)), _stream(x)))
    return q, s


def peer_silu_mul_quant(comm: PeerComm, gate_up: torch.Tensor, precise_div: bool = True,
                        round_silu: bool = False):
    """silu(gate)*up + per-token int8 of this GPU's [gate_r | up_r] slice (global absmax)."""
    assert gate_up.is_contiguous() and gate_up.dim() == 2
    m, i = gate_up.shape[0], gate_up.shape[1] // 2
    q = torch.empty((m, i), dtype=torch.int8, device=gate_up.device)
    s = torch.empty((m, 1), dtype=torch.float32, device=gate_up.device)
    if m and i:
        _native.check(_native.load().i8l_tp_silu_mul_quant(
            ctypes.byref(comm.desc), gate_up.data_ptr(), gate_up.stride(0), _ACT[gate_up.dtype],
            q.data_ptr(), q.stride(0), s.data_ptr(), m, i, int(bool(precise_div)), int(bool(round_silu)),
            _stream(gate_up)))
    return q, s


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

    comm: PeerComm | None = None

    def partial(self, a_q_shard) -> torch.Tensor:
        """This rank's int32 partial product [M, N] over its K/g slice."""
        return self.ops.mm_raw(a_q_shard, self.w)

    def __call__(self, a_q_shard, a_s, out_dtype=torch.bfloat16):
        """a_q_shard: this rank's int8 columns [M, K/g]; a_s: the GLOBAL per-token scale."""
        acc = self.partial(a_q_shard)
        if self.comm is not None and self.comm.fits(acc.shape[0], acc.shape[1] * 8):
            try:
                return peer_allreduce_dequant(self.comm, acc, a_s, self.w_s, out_dtype, self.bias)
            except _native.NotSupported:
                pass
        dist.all_reduce(acc, op=dist.ReduceOp.SUM, group=self.group)
        return self.ops.dequant(acc, a_s, self.w_s, out_dtype, self.bias)


def sharded_per_token_quant(x_shard, group=None, ops=None, comm: PeerComm | None = None):
    """Per-token int8 of a row split over the ranks (x_shard [M, K/g]), with the scale of
    the whole row: (q_shard, scale [M, 1]) identical to one GPU's on the full row."""
    if comm is not None and comm.fits(x_shard.shape[0], 16):
        return peer_quant_rows(comm, x_shard)
    ops = ops or CudaOps()
    amax = ops.absmax(x_shard)
    dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=group)
    return ops.quant(x_shard, absmax=amax)


def sharded_silu_mul_quant(gate_up_shard, round_silu: bool = False, group=None, ops=None,
                           comm: PeerComm | None = None):
    """SiLU-and-mul + per-token int8 of gate||up columns split over the ranks
    (gate_up_shard = [gate_r | up_r], [M, 2 I/g]), with the whole row's scale."""
    if comm is not None and comm.fits(gate_up_shard.shape[0], 16):
        return peer_silu_mul_quant(comm, gate_up_shard, round_silu=round_silu)
    ops = ops or CudaOps()
    amax = ops.silu_absmax(gate_up_shard, round_silu)
    dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=group)
    return ops.silu_quant(gate_up_shard, round_silu, absmax=amax)
