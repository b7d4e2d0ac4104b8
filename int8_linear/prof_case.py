"""Small, self-contained GPU workloads for profiling the kernels (e.g. under ncu).

    python -m int8_linear.prof_case gemm M N K [--config bm,bn[,split[,cluster]]] [--iters 4]
    python -m int8_linear.prof_case sweep [--model qwen3-1.7b-vllm]      # every (layer, M) once
    python -m int8_linear.prof_case quant M [--kind norm|silu|plain]

Each runs a few warm-up launches first, so `ncu -s <skip> -c <count>` can pick
steady-state launches, and keeps the device footprint small (one weight per layer).
"""

from __future__ import annotations

import argparse

import torch

from int8_linear import fused_quant as fq
from int8_linear import set_pdl, w8a8_mm
from int8_linear.kernel import Config
from int8_linear.shapes import SHAPES

SWEEP_M = [1, 2, 4, 8, 16, 17, 32, 64, 128, 256, 1024, 4096]


def _ints(shape, g):
    return torch.randint(-127, 128, shape, dtype=torch.int8, device="cuda", generator=g)


def gemm(m: int, n: int, k: int, cfg: Config | None, iters: int) -> None:
    g = torch.Generator(device="cuda").manual_seed(0)
    a = _ints((m, k), g)
    ws = [_ints((n, k), g) for _ in range(2)]
    sa = torch.rand((m, 1), device="cuda", generator=g) * 1e-2 + 1e-3
    sb = torch.rand((n, 1), device="cuda", generator=g) * 1e-3 + 1e-4
    for i in range(iters):
        w8a8_mm(a, ws[i % 2].t(), sa, sb, torch.bfloat16, config=cfg)
    torch.cuda.synchronize()


def sweep(model: str) -> None:
    g = torch.Generator(device="cuda").manual_seed(0)
    for _, k, n in SHAPES[model]:
        w = _ints((n, k), g)
        sb = torch.rand((n, 1), device="cuda", generator=g) * 1e-3 + 1e-4
        for m in SWEEP_M:
            a = _ints((m, k), g)
            sa = torch.rand((m, 1), device="cuda", generator=g) * 1e-2 + 1e-3
            w8a8_mm(a, w.t(), sa, sb, torch.bfloat16)
        torch.cuda.synchronize()


def quant(m: int, kind: str, iters: int) -> None:
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn((m, 2048), device="cuda", generator=g).to(torch.bfloat16)
    r = torch.randn((m, 2048), device="cuda", generator=g).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(2048, device="cuda", generator=g)).to(torch.bfloat16)
    gu = torch.randn((m, 12288), device="cuda", generator=g).to(torch.bfloat16)
    for _ in range(iters):
        if kind == "norm":
            fq.add_rmsnorm_quant(x, r, gamma, 1e-6)
        elif kind == "silu":
            fq.silu_mul_quant(gu, True, True)
        else:
            fq.per_token_quant(x)
    torch.cuda.synchronize()


def main() -> None:
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="what", required=True)
    p = sub.add_parser("gemm")
    p.add_argument("m", type=int)
    p.add_argument("n", type=int)
    p.add_argument("k", type=int)
    p.add_argument("--config", default=None)
    p.add_argument("--iters", type=int, default=4)
    p = sub.add_parser("sweep")
    p.add_argument("--model", default="qwen3-1.7b-vllm")
    p = sub.add_parser("quant")
    p.add_argument("m", type=int)
    p.add_argument("--kind", default="norm", choices=["norm", "silu", "plain"])
    p.add_argument("--iters", type=int, default=4)
    ap.add_argument("--pdl", action="store_true", help="programmatic dependent launch")
    args = ap.parse_args()
    set_pdl(args.pdl)
    if args.what == "gemm":
        cfg = None
        if args.config:
            f = [int(v) for v in args.config.split(",")]
            cfg = Config(f[0], f[1], split=f[2] if len(f) > 2 else 0, cluster=f[3] if len(f) > 3 else 0)
        gemm(args.m, args.n, args.k, cfg, args.iters)
    elif args.what == "sweep":
        sweep(args.model)
    else:
        quant(args.m, args.kind, args.iters)


if __name__ == "__main__":
    main()
