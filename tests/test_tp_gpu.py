"""Tensor parallelism: the TP stand-in decoder (NCCL collectives or this library's NVLink
exchange kernels) and each exchange kernel give exactly the one-GPU results.  Runs on 2
GPUs (I8L_TP_WORLD=4 or 8 for more); skipped when the box has fewer."""

from __future__ import annotations

import datetime
import os
import tempfile

import pytest
import torch

pytestmark = pytest.mark.gpu
WORLD = int(os.environ.get("I8L_TP_WORLD", "2"))


def _rendezvous_file():
    """A fresh file for the process group's rendezvous (no TCP port to race for)."""
    fd, path = tempfile.mkstemp(prefix="i8l_tp_")
    os.close(fd)
    os.unlink(path)
    return path


def _init(rank, path):
    import torch.distributed as dist

    os.environ.update(NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"file://{path}", rank=rank, world_size=WORLD,
                            device_id=dev, timeout=datetime.timedelta(seconds=120))
    return dev


def _worker(rank, path, m, mode, q):
    import torch.distributed as dist

    from int8_linear import set_pdl
    from int8_linear.standin import StandinDecoder, TPStandinDecoder
    from int8_linear.tp import PeerComm

    dev = _init(rank, path)
    comm = None
    try:
        set_pdl(True)
        comm = (PeerComm(device=dev, two_shot_rows=1 if mode == "peer2" else 0)
                if mode.startswith("peer") else None)
        tpd = TPStandinDecoder(m, rank, WORLD, layers=3, device=dev, comm=comm)
        eager = tpd.step()
        g = tpd.capture()
        outs_ok = True
        for _ in range(3):          # replays advance the exchange epochs
            g.replay()
            torch.cuda.synchronize()
            outs_ok = outs_ok and torch.equal(tpd.out, eager)
        ref = StandinDecoder(m, layers=3, device=dev).step() if rank == 0 else None
        same = bool(torch.equal(eager, ref)) if rank == 0 else True
        del g, tpd
        q.put((rank, outs_ok, same))
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


def _run(target, *args):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    path = _rendezvous_file()
    procs = [ctx.Process(target=target, args=(r, path, *args, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(WORLD)]
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    return res


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason=f"needs {WORLD} GPUs")
@pytest.mark.parametrize("mode", ["nccl", "peer", "peer2"])
@pytest.mark.parametrize("m", [1, 16])
def test_tp_standin_equals_one_gpu(m, mode):
    """peer2: the NVLink exchange kernels with the row-parallel sums forced two-shot."""
    for rank, ok, same in _run(_worker, m, mode):
        assert ok, f"rank {rank}: graph replay differs from eager"
        assert same, f"rank {rank}: TP output differs from the one-GPU stand-in"


def _ops_worker(rank, path, two_shot, q):
    import torch.distributed as dist

    from int8_linear import fused_quant as fq
    from int8_linear import tp
    from int8_linear.kernel import w8a8_mm

    dev = _init(rank, path)
    comm = None
    fails = []
    try:
        comm = tp.PeerComm(device=dev, two_shot_rows=1 if two_shot else -1)
        one = torch.ones(1, device=dev)
        for m, k, n in [(1, 2048, 2048), (5, 1024, 4096), (64, 6144, 2048), (200, 512, 1024)]:
            g = torch.Generator(device=dev).manual_seed(m * 7 + n)
            a = torch.randint(-127, 128, (m, k), dtype=torch.int8, device=dev, generator=g)
            w = torch.randint(-127, 128, (n, k), dtype=torch.int8, device=dev, generator=g)
            sa = torch.rand((m, 1), device=dev, generator=g) * 1e-2 + 1e-3
            sb = torch.rand((n, 1), device=dev, generator=g) * 1e-3 + 1e-4
            bias = (torch.randn(n, device=dev, generator=g) * 0.01).to(torch.bfloat16)
            res = torch.randn((m, n), device=dev, generator=g).to(torch.bfloat16)
            gamma = (1 + 0.1 * torch.randn(n, device=dev, generator=g)).to(torch.bfloat16)
            full = w8a8_mm(a, w.t(), sa, sb, torch.bfloat16, bias)
            ks = k // WORLD
            acc = w8a8_mm(a[:, rank * ks:(rank + 1) * ks].contiguous(),
                          w[:, rank * ks:(rank + 1) * ks].contiguous().t(), one, one, raw=True)
            for rep in range(3):   # repeated calls: epochs and parities advance
                got = tp.peer_allreduce_dequant(comm, acc, sa, sb, torch.bfloat16, bias)
                if not torch.equal(got, full):
                    fails.append(("allreduce_dequant", m, k, n, rep))
            q0, s0, r0 = fq.add_rmsnorm_quant(full, res, gamma, 1e-6)
            h = torch.empty_like(full)
            q1, s1, r1 = tp.peer_allreduce_add_rmsnorm_quant(comm, acc, sa, sb, bias, res, gamma, 1e-6,
                                                             h_out=h)
            if not (torch.equal(q0, q1) and torch.equal(s0, s1) and torch.equal(r0, r1) and torch.equal(h, full)):
                fails.append(("allreduce_norm", m, k, n))
            x = torch.randn((m, 2 * n), device=dev, generator=g).to(torch.bfloat16) * 3
            cs = n // WORLD   # this rank's column slice of a row of n values
            xs = x[:, :n][:, rank * cs:(rank + 1) * cs]
            qf2, sf2 = fq.per_token_quant(x[:, :n])
            qp, sp = tp.peer_quant_rows(comm, xs)
            if not (torch.equal(qp, qf2[:, rank * cs:(rank + 1) * cs]) and torch.equal(sp, sf2)):
                fails.append(("quant_rows", m, n))
            i = n // WORLD
            gs = torch.cat([x[:, :n][:, rank * i:(rank + 1) * i], x[:, n:][:, rank * i:(rank + 1) * i]], 1)
            for rs in (False, True):
                qs_, ss_ = fq.silu_mul_quant(x.contiguous(), True, rs)
                qp, sp = tp.peer_silu_mul_quant(comm, gs.contiguous(), round_silu=rs)
                if not (torch.equal(qp, qs_[:, rank * i:(rank + 1) * i]) and torch.equal(sp, ss_)):
                    fails.append(("silu_mul_quant", m, n, rs))
        torch.cuda.synchronize()
        from int8_linear import _native
        status = _native.read_status()
        q.put((rank, fails, status))
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason=f"needs {WORLD} GPUs")
@pytest.mark.parametrize("two_shot", [False, True])
def test_peer_exchange_ops_equal_one_gpu(two_shot):
    """Every exchange kernel on two GPUs gives what one GPU gives on the whole row, with
    the row-parallel sums one-shot and two-shot (reduce-scatter + all-gather)."""
    for rank, fails, status in _run(_ops_worker, two_shot):
        assert status == 0, f"rank {rank}: status word {status}"
        assert not fails, f"rank {rank}: {fails}"
