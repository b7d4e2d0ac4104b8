"""Per-shape tile tuner for B200: writes int8_linear/tuned_configs.json.

    python -m int8_linear.tune [--shapes qwen3-1.7b-vllm llama-3-8b] [--m 1 2 4 ...]
                               [--tp 1 2 4 8] [--out PATH] [--context gemm|decode]

Same table format as the reference's tuned_configs.json (read by tuned_config,
int8_linear/kernel.py):  {device name: {"KxN": {"M": {"config": {...}, "graph_us": t}}}}.
For every (K, N, M) each candidate tiling is timed as a CUDA graph of back-to-back
launches, each on its own copy of the weight, the copies together at least twice the L2
and the L2 flushed before each timed replay (L2-cold, as in a decode step that streams
every layer's weights), with programmatic dependent launch on; the fastest goes into
the table.  A candidate whose int32 product differs from the default tiling's is
rejected (all tilings must give identical bits).  --tp N also tunes the per-GPU shards
of a tensor-parallel split (column shards N/g of qkv and gate_up, row shards K/g of
o_proj and down).

--context decode (the default) times each candidate the way a decode step runs it: every
GEMM follows the add+RMSNorm+quant kernel that produces its int8 activations (the time of
that quantiser alone is subtracted).  --context gemm times GEMMs back to back.  On the
28-layer stand-in decode step, tables tuned in decode context with L2-cold weights
predicted the fastest tilings; tables tuned with 8 rotated copies (67 MB for a
2048 x 4096 weight, inside the 126 MB L2) picked narrow tiles that were slower there.
"""

from __future__ import annotations

import argparse
import json
import statistics
from dataclasses import asdict

import torch

from int8_linear import _native
from int8_linear import fused_quant as fq
from int8_linear.kernel import GEMV_TOKENS, TOKEN_TILES, TUNED_PATH, Config, NotSupported, default_config, w8a8_mm
from int8_linear.shapes import SHAPES

M_DEFAULT = [1, 2, 4, 8, 16, 17, 32, 64, 128, 256, 1024, 4096]
COPIES = 8            # fewest weight copies per graph
L2_BYTES = 126 << 20  # B200


def pool_size(nbytes: int) -> int:
    """Weight copies one graph rotates through: at least COPIES, and together at least
    twice the L2, so that no launch finds its weight left in L2 by an earlier one."""
    return max(COPIES, -(-2 * L2_BYTES // nbytes))


_flush: torch.Tensor | None = None


def flush_l2() -> None:
    global _flush
    if _flush is None:
        _flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device="cuda")
    _flush.zero_()


def candidates(m: int, n: int, k: int, sms: int) -> list[Config]:
    """Tilings worth timing for this shape (deduplicated, each B200-valid)."""
    out: list[Config] = [default_config(m, n, k)]
    cdiv = lambda a, b: -(-a // b)  # noqa: E731
    if m <= 256:
        holding = [t for t in TOKEN_TILES if t >= m][:1]
        smaller = [t for t in TOKEN_TILES if t < m and t >= m / 4][-1:]
        for tn in holding + smaller:
            tiles = cdiv(n, 128) * cdiv(m, tn)
            out += [Config(tn, 128, split=1), Config(tn, 128, split=1, ctas=tiles),
                    Config(tn, 128, split=2)]
            if tn <= 64:
                out += [Config(tn, 128, split=3)] + [Config(tn, 128, split=3, cluster=c) for c in (2, 3, 4, 8)]
                # activation by plain loads after the dependency wait (where it fits)
                out += [Config(tn, 128, split=3, cluster=c, act=a) for c in (2, 3, 4, 8) for a in (1, 2)]
                out += [Config(tn, 128, split=1, ctas=tiles, act=2)]
            if m <= 16:   # narrow tiles: the weight on the MMA's N side (256 rows per MMA)
                out += [Config(128, 256, split=3, cluster=c) for c in (1, 2, 3, 4, 6, 8)]
            if m <= 32:   # plain versus TMA stores for the few output rows
                out += [Config(tn, 128, split=3, cluster=c, store=1) for c in (2, 4)]
                out += [Config(tn, 128, split=1, store=1), Config(tn, 128, split=2, store=2)]
    if m <= 16:   # CUDA-core tiles: whole output columns per CTA, no split-K
        mt = next(t for t in GEMV_TOKENS if t >= m)
        out += [Config(mt, 0, split=5), Config(mt, 0, split=5, ctas=2 * sms),
                Config(mt, 0, split=5, stages=16)]
    if 16 < m <= 512:   # cluster split-K with the weight on the MMA's N side (128 tokens x 128/256)
        out += [Config(128, bn, split=3, cluster=c) for bn in (128, 256) for c in (2, 3, 4, 6, 8)]
    if 64 < m <= 256:   # cluster split-K on the 128- and 256-token swap tiles
        tn = next(t for t in TOKEN_TILES if t >= m)
        out += [Config(tn, 128, swap_ab=True, split=3, cluster=c) for c in (2, 3, 4, 6, 8)]
    if m >= 64:
        for bn in (128, 256):
            out += [Config(128, bn, split=1), Config(128, bn, split=2)]
    if m >= 256:   # CTA pairs: two SMs per 256 x 256 tile
        out += [Config(128, 256, split=4), Config(128, 256, split=4, group_m=16)]
    seen, uniq = set(), []
    for c in out:
        if c.name in seen:
            continue
        try:
            c.check()
        except NotSupported:
            continue
        seen.add(c.name)
        uniq.append(c)
    return uniq


def graph_us(fn, reps: int, windows: int = 5) -> float:
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(reps):
            fn()
    graph.replay()
    torch.cuda.synchronize()
    times = []
    for _ in range(windows):
        flush_l2()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b) * 1e3 / reps)
    del graph
    return statistics.median(times)


def rank_shape(k: int, n: int, ms: list[int], sms: int, context: str = "gemm") -> dict[int, list]:
    """Every valid candidate tiling of each batch size M, fastest first: {M: [(Config,
    µs), ...]}.  A candidate whose int32 product differs from the default tiling's raises."""
    g = torch.Generator(device="cuda").manual_seed(k * 31 + n)
    copies = pool_size(n * k)
    ws = [torch.randint(-127, 128, (n, k), dtype=torch.int8, device="cuda", generator=g)
          for _ in range(copies)]
    sb = torch.rand((n, 1), device="cuda", generator=g) * 1e-3 + 1e-4
    one = torch.ones(1, device="cuda")
    ranked = {}
    for m in ms:
        a = torch.randint(-127, 128, (m, k), dtype=torch.int8, device="cuda", generator=g)
        sa = torch.rand((m, 1), device="cuda", generator=g) * 1e-2 + 1e-3
        want = w8a8_mm(a, ws[0].t(), one, one, raw=True, config=default_config(m, n, k))
        x = torch.randn((m, k), device="cuda", generator=g).to(torch.bfloat16)
        gamma = torch.ones(k, device="cuda", dtype=torch.bfloat16)
        base = 0.0
        if context == "decode":
            base = graph_us(lambda: fq.add_rmsnorm_quant(x, None, gamma, 1e-6), copies)
        timed = []
        for cfg in candidates(m, n, k, sms):
            try:
                got = w8a8_mm(a, ws[0].t(), one, one, raw=True, config=cfg)
            except NotSupported:
                continue
            if not torch.equal(got, want):
                raise AssertionError(f"{cfg.name} differs from the default tiling at {m}x{k}x{n}")
            it = iter(range(1 << 40))

            def fn(cfg=cfg, it=it):
                if context == "decode":
                    q, s, _ = fq.add_rmsnorm_quant(x, None, gamma, 1e-6)
                    w8a8_mm(q, ws[next(it) % copies].t(), s, sb, torch.bfloat16, config=cfg)
                else:
                    w8a8_mm(a, ws[next(it) % copies].t(), sa, sb, torch.bfloat16, config=cfg)

            timed.append((cfg, graph_us(fn, copies) - base))
        assert timed, f"no candidate tiling runs {m}x{k}x{n}"
        ranked[m] = sorted(timed, key=lambda t: t[1])
    del ws
    torch.cuda.empty_cache()
    return ranked


def tune_shape(k: int, n: int, ms: list[int], sms: int, verbose: bool = True,
               context: str = "gemm") -> dict:
    """The table entries {"M": {"config", "graph_us"}} of one (K, N): the fastest candidate."""
    table = {}
    for m, timed in rank_shape(k, n, ms, sms, context).items():
        cfg, us = timed[0]
        table[str(m)] = {"config": asdict(cfg), "graph_us": round(us, 3)}
        if verbose:
            print(f"K={k:6d} N={n:6d} M={m:5d}: {cfg.name:40s} {us:9.2f} us", flush=True)
    return table


def shard_shapes(model: str, tp: int) -> list[tuple[int, int]]:
    """(K, N) per GPU: column shards for qkv and gate_up, row shards for o_proj and down."""
    out = []
    for label, k, n in SHAPES[model]:
        row_parallel = label.startswith(("o_proj", "down"))
        out.append((k // tp, n) if row_parallel else (k, n // tp))
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", nargs="*", default=["qwen3-1.7b-vllm", "llama-3-8b"])
    ap.add_argument("--m", nargs="*", type=int, default=M_DEFAULT)
    ap.add_argument("--tp", nargs="*", type=int, default=[1])
    ap.add_argument("--out", default=str(TUNED_PATH))
    ap.add_argument("--context", choices=["gemm", "decode"], default="decode",
                    help="time GEMMs back to back, or each after its activation quantiser")
    args = ap.parse_args()
    _native.set_pdl(True)
    dev = torch.cuda.get_device_name()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    try:
        with open(args.out) as f:
            tables = json.load(f)
    except FileNotFoundError:
        tables = {}
    table = tables.setdefault(dev, {})
    done = set()
    for model in args.shapes:
        for tp in args.tp:
            for k, n in shard_shapes(model, tp):
                if (k, n) in done:
                    continue
                done.add((k, n))
                table.setdefault(f"{k}x{n}", {}).update(tune_shape(k, n, args.m, sms, context=args.context))
                with open(args.out, "w") as f:
                    json.dump(tables, f, indent=1, sort_keys=True)
                    f.write("\n")
    print("wrote", args.out)


if __name__ == "__main__":
    main()
