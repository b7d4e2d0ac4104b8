"""Tensor-parallel orchestration (int8_linear/tp.py) with two gloo ranks on CPU.

The arithmetic is the CPU oracle's (oracle/); what is tested is the sharding of the
weights and activations and the collectives around the kernels: the row-parallel int32
SUM, the global-absmax MAX for split rows, the column all-gather.  Every TP result must
equal the one-process result bit for bit, as it does on GPUs with the CUDA kernels.
"""

from __future__ import annotations

import io
import os
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import gemm as og
from oracle import quant as oq
from oracle.numerics import round_bf16

WORLD = 2


class OracleOps:
    """The CPU oracle behind the ops interface of int8_linear.tp."""

    def mm_raw(self, a_q, w):
        return torch.from_numpy(og.exact(a_q.numpy(), w.numpy()))

    def dequant(self, acc, a_s, w_s, out_dtype, bias):
        v = og.epilogue_f32(acc.numpy(), a_s.numpy(), w_s.numpy(),
                            None if bias is None else bias.float().numpy())
        return torch.from_numpy(v).to(out_dtype)

    def mm(self, a_q, a_s, w, w_s, out_dtype, bias):
        return self.dequant(self.mm_raw(a_q, w), a_s, w_s, out_dtype, bias)

    def absmax(self, x):
        return x.float().abs().amax(-1)

    def quant(self, x, absmax=None):
        q, s = oq.quant_ieee(x.float().numpy(), None if absmax is None else absmax.numpy())
        return torch.from_numpy(q), torch.from_numpy(s)

    def _silu(self, gu):
        gu = gu.float().numpy()
        i = gu.shape[1] // 2
        g, u = gu[:, :i], gu[:, i:]
        a = (g / (np.float32(1.0) + np.exp(-g))).astype(np.float32)
        return round_bf16((a * u).astype(np.float32))

    def silu_absmax(self, gu, round_silu):
        return torch.from_numpy(np.abs(self._silu(gu)).max(-1).astype(np.float32))

    def silu_quant(self, gu, round_silu, absmax=None):
        q, s = oq.quant_ieee(self._silu(gu), None if absmax is None else absmax.numpy())
        return torch.from_numpy(q), torch.from_numpy(s)


def problem():
    g = torch.Generator().manual_seed(0)
    m, k, n = 5, 256, 96
    a_q = torch.randint(-127, 128, (m, k), dtype=torch.int8, generator=g)
    a_s = torch.rand((m, 1), generator=g) * 1e-2 + 1e-3
    w = torch.randint(-127, 128, (n, k), dtype=torch.int8, generator=g)
    w_s = torch.rand((n, 1), generator=g) * 1e-3 + 1e-4
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16)
    x = (torch.randn((m, k), generator=g) * 2).to(torch.bfloat16)
    gu = (torch.randn((m, 2 * k), generator=g) * 2).to(torch.bfloat16)
    return a_q, a_s, w, w_s, bias, x, gu


def _worker(rank, path, q):
    from int8_linear import tp

    dist.init_process_group("gloo", init_method=f"file://{path}", rank=rank, world_size=WORLD)
    try:
        ops = OracleOps()
        a_q, a_s, w, w_s, bias, x, gu = problem()
        res = {}
        # row-parallel: K split, int32 partials summed, dequantised once
        row = tp.RowParallelW8A8(tp.shard_cols_of(w, rank, WORLD), w_s, bias, ops=ops)
        res["row"] = row(tp.shard_cols_of(a_q, rank, WORLD), a_s)
        # column-parallel with merged segments (like gate||up) and all-gather
        col = tp.ColumnParallelW8A8(tp.shard_rows_of(w, rank, WORLD, parts=(64, 32)),
                                    tp.shard_rows_of(w_s, rank, WORLD, parts=(64, 32)),
                                    tp.shard_rows_of(bias, rank, WORLD, parts=(64, 32)), ops=ops)
        res["col"] = col(a_q, a_s, gather=True)
        # a row split over the ranks keeps the one-GPU per-token scale
        res["quant"] = tp.sharded_per_token_quant(tp.shard_cols_of(x, rank, WORLD), ops=ops)
        k = gu.shape[1] // 2
        gu_shard = torch.cat([tp.shard_cols_of(gu[:, :k], rank, WORLD),
                              tp.shard_cols_of(gu[:, k:], rank, WORLD)], dim=1)
        res["silu"] = tp.sharded_silu_mul_quant(gu_shard, ops=ops)
        # by value: tensors on a queue travel as shared-memory file descriptors, which
        # the parent cannot open once this process has exited
        buf = io.BytesIO()
        torch.save(res, buf)
        q.put((rank, buf.getvalue()))
    finally:
        dist.destroy_process_group()


def rendezvous_file():
    """A fresh file for the process group's rendezvous (no TCP port to race for)."""
    fd, path = tempfile.mkstemp(prefix="i8l_gloo_")
    os.close(fd)
    os.unlink(path)
    return path


@pytest.fixture(scope="module")
def results():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    path = rendezvous_file()
    procs = [ctx.Process(target=_worker, args=(r, path, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    out = {}
    import queue as _queue
    import time
    deadline = time.time() + 180
    while len(out) < WORLD and time.time() < deadline:
        try:
            r, blob = q.get(timeout=1)
            out[r] = torch.load(io.BytesIO(blob))
        except _queue.Empty:
            if any(p.exitcode not in (None, 0) for p in procs):
                break
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert len(out) == WORLD and all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return out


def test_row_parallel_equals_one_gpu(results):
    ops = OracleOps()
    a_q, a_s, w, w_s, bias, *_ = problem()
    want = ops.mm(a_q, a_s, w, w_s, torch.bfloat16, bias)
    for r in range(WORLD):
        assert torch.equal(results[r]["row"], want)


def test_column_parallel_gathers_the_full_output(results):
    ops = OracleOps()
    a_q, a_s, w, w_s, bias, *_ = problem()
    want = ops.mm(a_q, a_s, w, w_s, torch.bfloat16, bias)
    # merged segments (64 | 32) are sharded separately, so the gathered columns come
    # back grouped by rank: [seg0 r0, seg1 r0, seg0 r1, seg1 r1]
    cols = []
    for r in range(WORLD):
        cols += list(range(r * 32, (r + 1) * 32)) + list(range(64 + r * 16, 64 + (r + 1) * 16))
    for r in range(WORLD):
        assert torch.equal(results[r]["col"], want[:, cols])


def test_split_rows_quantise_like_the_whole_row(results):
    ops = OracleOps()
    *_, x, gu = problem()
    q_full, s_full = ops.quant(x)
    k = x.shape[1] // WORLD
    for r in range(WORLD):
        q, s = results[r]["quant"]
        assert torch.equal(s, s_full) and torch.equal(q, q_full[:, r * k:(r + 1) * k])
    q_full, s_full = ops.silu_quant(gu, False)
    i = gu.shape[1] // 2 // WORLD
    for r in range(WORLD):
        q, s = results[r]["silu"]
        assert torch.equal(s, s_full) and torch.equal(q, q_full[:, r * i:(r + 1) * i])
