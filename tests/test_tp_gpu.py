"""Tensor parallelism on 2 GPUs (NCCL): the TP stand-in decoder and the row-/column-
parallel linears give exactly the one-GPU results.  Needs two GPUs; skipped otherwise."""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu
WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, m, q):
    import torch.distributed as dist

    from int8_linear import set_pdl
    from int8_linear.standin import StandinDecoder, TPStandinDecoder

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        set_pdl(True)
        tpd = TPStandinDecoder(m, rank, WORLD, layers=3, device=dev)
        eager = tpd.step()
        g = tpd.capture()
        g.replay()
        torch.cuda.synchronize()
        ok = torch.equal(tpd.out, eager)
        ref = StandinDecoder(m, layers=3, device=dev).step() if rank == 0 else None
        same = bool(torch.equal(eager, ref)) if rank == 0 else True
        del g, tpd
        q.put((rank, ok, same))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs two GPUs")
@pytest.mark.parametrize("m", [1, 16])
def test_tp_standin_equals_one_gpu(m):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, m, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(WORLD)]
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    for rank, ok, same in res:
        assert ok, f"rank {rank}: graph replay differs from eager"
        assert same, f"rank {rank}: TP output differs from the one-GPU stand-in"
