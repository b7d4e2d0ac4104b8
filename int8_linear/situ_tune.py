"""Tile tuning inside the 28-layer stand-in decode step (B200): updates tuned_configs.json.

    python -m int8_linear.situ_tune [--batch 1,2,4,...] [--top 4] [--windows 5]
                                    [--rounds 3] [--out PATH] [--dry-run]

Timing each GEMM alone mispredicts the decode step: in the step every layer has its own
weights and a quantiser or norm sits between the GEMMs, so a tiling's weight prefetch
has less to hide behind, and its footprint decides what the next kernel can overlap.
The reference makes the same finding and tunes in a stand-in (bench/situ_tune.py:
224-264); this follows its procedure on this library's stand-in (int8_linear/standin.py):

for each decode batch M, start from the table's tilings of the four linears (qkv, o_proj,
gate_up, down).  One pass over the linears: each tries its current tiling, the untuned
default and the `top` fastest candidates of the per-layer timing in decode context
(int8_linear/tune.py rank_shape), each in a fresh capture of the whole step with the
other three fixed, and keeps the fastest.  The chosen set is then timed against the
starting set in alternating fresh captures, and written to the table only if it is at
least 1% faster; its entries carry "stand_in_us" (µs per decoder layer) instead of
"graph_us".  Every tiling gives the same bits, so only speed is at stake.

The reference first checks its stand-in against two served vLLM runs; those runs need
the W8A8 checkpoint, which is not available here, so that check is left out.
"""

from __future__ import annotations

import argparse
import json
import statistics
from dataclasses import asdict
from typing import Callable

import torch

from int8_linear.kernel import TUNED_PATH, Config, choose_config, default_config

ACCEPT = 0.01
BATCHES = [1, 2, 4, 8, 16, 17, 32, 64, 128, 256]


# ------------------------------------------------------------------ selection (host only)
def layer_options(current: Config, default: Config, ranked: list[Config], top: int) -> list[Config]:
    """The tilings one linear tries: its current one, the untuned default, then the `top`
    fastest of the per-layer ranking, without repeats, in that order."""
    return list(dict.fromkeys([current, default, *ranked[:top]]))


def coordinate_pass(start: dict[str, Config], options: dict[str, list[Config]],
                    measure: Callable[[dict[str, Config]], float]) -> tuple[dict[str, Config], list]:
    """One pass over the linears in `start`'s order: each tries its options with the others
    fixed at the best found so far and keeps the fastest.  Returns the chosen tilings and
    the trials [(name, config, µs)]."""
    current = dict(start)
    trials = []
    for name in start:
        best = None
        for cfg in options[name]:
            us = measure({**current, name: cfg})
            trials.append((name, cfg, us))
            if best is None or us < best[1]:
                best = (cfg, us)
        current[name] = best[0]
    return current, trials


def accept(start_us: float, chosen_us: float, margin: float = ACCEPT) -> bool:
    """Keep a new set only when it is faster than the start by at least `margin`."""
    return chosen_us < start_us * (1.0 - margin)


def write_entries(table: dict, shapes: dict[str, tuple[int, int]], m: int,
                  chosen: dict[str, Config], us_per_layer: float) -> None:
    """Put the chosen tilings into a device's table as the entries of batch bucket M."""
    for name, (k, n) in shapes.items():
        table.setdefault(f"{k}x{n}", {})[str(m)] = {"config": asdict(chosen[name]),
                                                    "stand_in_us": round(us_per_layer, 3)}


# ------------------------------------------------------------------ timing (GPU)
_flush: torch.Tensor | None = None


def step_us(decoder, windows: int) -> float:
    """µs per decoder layer of one replay of a fresh capture (median of `windows`, L2
    flushed before each)."""
    global _flush
    from int8_linear.standin import LAYERS

    if _flush is None:
        _flush = torch.empty(2 * (126 << 20), dtype=torch.uint8, device="cuda")
    graph = decoder.capture()
    graph.replay()
    torch.cuda.synchronize()
    times = []
    for _ in range(windows):
        _flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b) * 1e3 / LAYERS)
    decoder.graph = None
    del graph
    return statistics.median(times)


def alternating(decoder, sets: dict[str, dict[str, Config]], rounds: int, windows: int) -> dict:
    """Median µs per layer of each set of tilings over `rounds` alternating fresh captures."""
    runs: dict[str, list[float]] = {label: [] for label in sets}
    for _ in range(rounds):
        for label, configs in sets.items():
            decoder.configs = dict(configs)
            runs[label].append(step_us(decoder, windows))
    return {label: round(statistics.median(v), 3) for label, v in runs.items()}


def tune_batch(m: int, top: int, windows: int, rounds: int, sms: int, verbose: bool = True) -> dict:
    from int8_linear.standin import SHAPES, StandinDecoder
    from int8_linear.tune import rank_shape

    start = {name: choose_config(m, n, k) for name, (k, n) in SHAPES.items()}
    options = {}
    for name, (k, n) in SHAPES.items():
        ranked = [cfg for cfg, _ in rank_shape(k, n, [m], sms, context="decode")[m]]
        options[name] = layer_options(start[name], default_config(m, n, k), ranked, top)
    decoder = StandinDecoder(m)

    def measure(configs: dict[str, Config]) -> float:
        decoder.configs = dict(configs)
        return step_us(decoder, windows)

    chosen, trials = coordinate_pass(start, options, measure)
    entry = {"batch": m, "start": {k: v.name for k, v in start.items()},
             "chosen": {k: v.name for k, v in chosen.items()},
             "trials": [(name, cfg.name, round(us, 3)) for name, cfg, us in trials], "kept": False}
    if chosen != start:
        t = alternating(decoder, {"start": start, "chosen": chosen}, max(rounds, 3), windows)
        entry["confirm_us"] = t
        entry["kept"] = accept(t["start"], t["chosen"])
    entry["chosen_configs"] = chosen
    del decoder
    torch.cuda.empty_cache()
    if verbose:
        changed = {k: f"{entry['start'][k]} -> {entry['chosen'][k]}" for k in start
                   if entry["start"][k] != entry["chosen"][k]}
        print(f"batch {m}: {changed or 'no change'}; confirm {entry.get('confirm_us')}; "
              f"kept {entry['kept']}", flush=True)
    return entry


def main() -> None:
    from int8_linear import _native
    from int8_linear.standin import SHAPES

    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--batch", default=",".join(map(str, BATCHES)))
    ap.add_argument("--top", type=int, default=4, help="fastest per-layer candidates tried per linear")
    ap.add_argument("--windows", type=int, default=5)
    ap.add_argument("--rounds", type=int, default=3)
    ap.add_argument("--out", default=str(TUNED_PATH))
    ap.add_argument("--report", default=None, help="also write the trials as JSON here")
    ap.add_argument("--dry-run", action="store_true", help="tune and report, write no table")
    args = ap.parse_args()
    _native.set_pdl(True)
    dev = torch.cuda.get_device_name()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    try:
        with open(args.out) as f:
            tables = json.load(f)
    except FileNotFoundError:
        tables = {}
    results = []
    for m in (int(x) for x in args.batch.split(",")):
        entry = tune_batch(m, args.top, args.windows, args.rounds, sms)
        chosen = entry.pop("chosen_configs")
        if entry["kept"] and not args.dry_run:
            write_entries(tables.setdefault(dev, {}), SHAPES, m, chosen, entry["confirm_us"]["chosen"])
            with open(args.out, "w") as f:
                json.dump(tables, f, indent=1, sort_keys=True)
                f.write("\n")
        results.append(entry)
    if args.report:
        with open(args.report, "w") as f:
            json.dump(results, f, indent=1)
    print("kept:", [e["batch"] for e in results if e["kept"]])


if __name__ == "__main__":
    main()
