"""Benchmark of the W8A8 hot path on B200; rank 0 prints one short JSON line last.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference|reference-triton]
                    [--model qwen3-1.7b-vllm|llama-3-8b] [--no-standin] [--no-e2e] [--no-pdl]
                    [--out FILE] [--detail FILE]
    python bench.py --case gemm|sweep|quant|dequant|standin [--shape ...] [...]   (profiling workloads)

Workload: the per-layer sweep at the Qwen3-1.7B shapes vLLM runs
(qkv 2048x4096, o_proj 2048x2048, gate_up 2048x12288, down 6144x2048), every M in
{1,2,4,8,16,17,32,64,128,256,1024,4096}, with and without a bf16 bias: 96 GEMMs.
Inputs are generated as in config 0 (bf16 N(0,1) activations and N(0,0.02) weights,
quantised per row to int8).  Before anything is timed every case runs once into an
output filled with NaN and is checked against the reference's float64 layer and,
bit for bit, against the fp32 epilogue order (`checked` in the line).  One step runs
every case R=8 times back to back from CUDA graphs, each launch on its own weight copy
from a per-layer pool holding at least twice the 126 MB L2, so weights are always
L2-cold.  `value` is microseconds per sweep (one GEMM of each case), device time.
`e2e` is the same sweep through the public API w8a8_mm, eagerly, with each step's int8
activations and scales copied in from pinned host memory and every output copied back.

The final line keeps to a few KB (only the tail of stdout is read); the per-shape
table, the L2-warm timings and the full quantiser table go to the --detail file
(default: bench_detail_n<N>.json in the run's output folder, see detail_path).

Under torchrun (N > 1) each rank runs its column shard (N/g output columns) of every
layer, independently; the NCCL all-gather of the shards is timed separately and
reported as `allgather_us_per_sweep`.  The config-2 (Llama-3-8B) sweep is run the same
way and reported as `config2_us_per_sweep`, and the stand-in decoder runs tensor
parallel in both exchange modes.

--impl reference times the reference's CPU implementation of the path on this host's
cores: the float64 torch layer of bench/bench_linear.py:164-165 (restated in
oracle/gemm.py layer_f64_torch) over the whole sweep, every M and N, on rank 0 only.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "W8A8 GEMM µs & roofline % per (M,K,N); stand-in decode µs/layer at bs 1–128"
M_SWEEP = [1, 2, 4, 8, 16, 17, 32, 64, 128, 256, 1024, 4096]
QUANT_M = [1, 16, 64, 128, 1024, 4096]    # BASELINE config 3 batch sizes timed
QUANT_M_LINE = ["1", "128", "4096"]       # the ones the final line carries
STANDIN_BATCHES = [1, 2, 4, 8, 16, 32, 64, 128]
COPIES = 8          # launches per shape per step, each on its own weight copy
L2_BYTES = 126 << 20
LINE_LIMIT = 4000   # bytes of the final JSON line


def pool_size(nbytes: int) -> int:
    """Copies of one weight to rotate through: together at least twice the L2, in whole
    windows of COPIES, so no launch finds its weight left in L2 by an earlier one."""
    n = max(COPIES, -(-2 * L2_BYTES // nbytes))
    return -(-n // COPIES) * COPIES


_FLUSH = None


def flush_l2():
    """Write a buffer twice the L2's size (evicts every weight and activation)."""
    import torch

    global _FLUSH
    if _FLUSH is None:
        _FLUSH = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device="cuda")
    _FLUSH.zero_()


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference", "reference-triton", "reference-triton-child"],
                    default="ours")
    ap.add_argument("--model", default="qwen3-1.7b-vllm")
    ap.add_argument("--no-standin", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-pdl", action="store_true", help="launch without programmatic dependent launch")
    ap.add_argument("--no-config2", action="store_true", help="skip the config-2 (Llama-3-8B) sweep")
    ap.add_argument("--out", default=None, help="also write the final JSON line to this file")
    ap.add_argument("--detail", default=None, help="where the per-shape tables go")
    # profiling workloads (small, self-contained; for ncu captures)
    ap.add_argument("--case", choices=["gemm", "sweep", "quant", "dequant", "standin"], default=None)
    ap.add_argument("--shape", default=None, help="gemm: M,N,K; quant: M; standin: batch")
    ap.add_argument("--config", default=None, help="gemm: bm,bn[,split[,cluster]]")
    ap.add_argument("--kind", default="norm", choices=["norm", "silu", "plain"])
    ap.add_argument("--iters", type=int, default=4)
    return ap.parse_args()


def peaks(int8_tops: float | None = None) -> dict:
    p = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        p = {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    if int8_tops:
        p["int8_tops"], p["int8_source"] = int8_tops, "measured int8 on this box (int8_tops_measured)"
    else:
        p["int8_tops"], p["int8_source"] = 2.0 * p["bf16_tflops"], p["source"] + " bf16 x2"
    return p


def layers_for(model: str):
    from int8_linear.shapes import SHAPES

    names = {"qwen3-1.7b-vllm": ["qkv", "o_proj", "gate_up", "down"],
             "llama-3-8b": ["qkv", "o_proj", "gate_up", "down"]}[model]
    return [(nm, k, n) for nm, (_, k, n) in zip(names, SHAPES[model])]


def alg_bytes(m, k, n, bias) -> int:
    """Bytes the GEMM must move at least once: A, W, scales, bias, bf16 output."""
    return m * k + n * k + 4 * m + 4 * n + (2 * n if bias else 0) + 2 * m * n


def cpu_model() -> str:
    try:
        for ln in Path("/proc/cpuinfo").read_text().splitlines():
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region.
    Entering waits (up to 3 s) for nvidia-smi's first sample, so sampling runs before the
    region starts; leaving waits (up to 1 s) for a sample taken after the region began, so
    a region shorter than the 50 ms interval still has one."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.lines: list[str] = []
        self.start = 0

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.dev}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            t0 = time.time()
            while not self.lines and time.time() - t0 < 3.0 and self.proc.poll() is None:
                time.sleep(0.01)
            self.start = len(self.lines)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            t0 = time.time()
            while len(self.lines) <= self.start and time.time() - t0 < 1.0 and self.proc.poll() is None:
                time.sleep(0.01)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines[self.start:]:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for nm, val in zip(names, parts[4:8]):
                if val.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------- setup
def quant_rows_t(x):
    """Per-row symmetric int8 (the operand generation of bench/bench_linear.py:146-150)."""
    import torch

    scale = x.float().abs().amax(dim=1, keepdim=True).clamp_min(1e-8) / 127.0
    return (x.float() / scale).round().clamp(-127, 127).to(torch.int8), scale


def build_operands(model, world, rank, dev):
    import torch

    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    layers = []
    for name, k, n in layers_for(model):
        assert n % world == 0, f"{name}: N={n} does not split over {world} GPUs"
        nl = n // world
        copies = []
        for _ in range(pool_size(nl * k)):
            w = (torch.randn((nl, k), generator=g, device=dev) * 0.02).to(torch.bfloat16)
            wq, ws = quant_rows_t(w)
            del w
            copies.append((wq, ws))
        bias = (torch.randn((nl,), generator=g, device=dev) * 0.01).to(torch.bfloat16)
        layers.append({"name": name, "k": k, "n": n, "nl": nl, "copies": copies, "bias": bias})
    acts = {}
    for k in sorted({lay["k"] for lay in layers}):
        for m in M_SWEEP:
            a = torch.randn((m, k), generator=g, device=dev).to(torch.bfloat16)
            acts[(m, k)] = quant_rows_t(a)
    return layers, acts


def sweep_cases(layers):
    return [(lay, m, bias) for bias in (False, True) for lay in layers for m in M_SWEEP]


_SIDE = None


def capture(fn):
    """CUDA graph of fn, after one warm-up call on a side stream (one stream for all
    captures, so the library keeps a single split-K workspace for them)."""
    import torch

    global _SIDE
    if _SIDE is None:
        _SIDE = torch.cuda.Stream()
    side = _SIDE
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    return graph


def time_graph(graph, windows=5, flush=True):
    """Median µs of `windows` replays, L2 flushed before each (outside the timed span)
    unless flush is False."""
    import torch

    graph.replay()
    torch.cuda.synchronize()
    ts = []
    for _ in range(windows):
        if flush:
            flush_l2()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b) * 1e3)
    return statistics.median(ts)


def launcher(acts, lay, m, bias, copies):
    """The graphed body of one case: w8a8_mm of the case's activation on each weight copy."""
    import torch

    from int8_linear import w8a8_mm

    a_q, a_s = acts[(m, lay["k"])]
    b = lay["bias"] if bias else None

    def fn():
        for wq, ws in copies:
            w8a8_mm(a_q, wq.t(), a_s, ws, torch.bfloat16, b)
    return fn


def capture_sweep(layers, acts, cases):
    """Per-case graphs: COPIES launches on distinct weight copies, each case on the next
    window of its layer's pool (L2-cold in the timed region too, where the cases of a
    layer run back to back)."""
    graphs, window = [], {}
    for lay, m, bias in cases:
        w0 = window.get(lay["name"], 0)
        window[lay["name"]] = (w0 + COPIES) % len(lay["copies"])
        graphs.append(capture(launcher(acts, lay, m, bias, lay["copies"][w0:w0 + COPIES])))
    return graphs


# ------------------------------------------------------------------- output checks
def check_case(a_q, a_s, wq, ws, bias) -> tuple[bool, float]:
    """Runs w8a8_mm once into an output filled with NaN and compares it with (1) the fp32
    epilogue order of the reference kernel (int8_linear/kernel.py:109-120: f32(acc)*sa,
    *sb, +bias, one rounding), bit for bit, and (2) the reference's float64 layer
    (bench/bench_linear.py:164-165), by the relative error its check uses
    (bench_linear.py:185-192).  The int32 product is a float64 GEMM of int8 values, exact
    in any order.  Returns (bit-exact, max relative error)."""
    import torch

    from int8_linear import w8a8_mm

    m, n = a_q.shape[0], wq.shape[0]
    out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=a_q.device)
    w8a8_mm(a_q, wq.t(), a_s, ws, torch.bfloat16, bias, out=out)
    acc64 = a_q.double() @ wq.double().t()
    v = acc64.to(torch.int32).to(torch.float32) * a_s.reshape(-1, 1)
    v = v * ws.reshape(1, -1)
    if bias is not None:
        v = v + bias.float().reshape(1, -1)
    exact = torch.equal(out.view(torch.int16), v.to(torch.bfloat16).view(torch.int16))
    term = acc64 * a_s.double().reshape(-1, 1) * ws.double().reshape(1, -1)
    ref = term + bias.double().reshape(1, -1) if bias is not None else term
    scale = torch.maximum(ref.abs(), term.abs()).clamp_min(1e-6)
    rel = ((out.double() - ref).abs() / scale).max().item()
    return exact, rel


def check_sweep(layers, acts, cases) -> dict:
    import torch

    ok = exact = 0
    worst = 0.0
    for lay, m, bias in cases:
        a_q, a_s = acts[(m, lay["k"])]
        wq, ws = lay["copies"][0]
        e, rel = check_case(a_q, a_s, wq, ws, lay["bias"] if bias else None)
        exact += int(e)
        ok += int(e and rel <= 1e-2)
        worst = max(worst, rel)
    torch.cuda.synchronize()
    return {"checked": f"{ok}/{len(cases)}", "bit_exact": exact, "max_rel_err_f64": float(f"{worst:.3g}")}


# ------------------------------------------------------------------- int8 peak
def int8_peak_probe(dev) -> dict:
    """Dense int8 throughput at 8192^3, best of 10 (CUDA events): torch._int_mm (cuBLASLt)
    and this library's w8a8_mm (int32 out, the library's tile).  The larger is the tensor
    roofline's peak."""
    import torch

    from int8_linear import w8a8_mm

    n = 8192
    g = torch.Generator(device=dev).manual_seed(7)
    a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev, generator=g)
    b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev, generator=g)
    sa = torch.ones((n, 1), device=dev)
    out = {}

    def best(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e-3)
        return round(2.0 * n ** 3 / min(ts) / 1e12, 1)

    try:
        out["torch_int_mm"] = best(lambda: torch._int_mm(a, b.t()))
    except RuntimeError as e:  # noqa: BLE001
        out["torch_int_mm"] = None
        out["torch_int_mm_error"] = str(e).splitlines()[0][:120]
    o32 = torch.empty((n, n), dtype=torch.int32, device=dev)
    out["ours_i32"] = best(lambda: w8a8_mm(a, b.t(), sa, sa, raw=True, out=o32))
    out["peak"] = max(v for v in (out.get("torch_int_mm"), out["ours_i32"]) if v)
    del a, b, o32
    torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------------- tie counts
def tie_counts(dev) -> dict:
    """BASELINE config 3 at M=4096: our fused quantisers against the reference's torch
    references (tests/test_fused_quant.py:26-51, restated here in torch on the GPU as the
    reference's test runs them): how many int8 values differ (each by one step, at a
    rounding tie or a boundary that a different summation order moves), and the largest
    difference."""
    import torch

    from int8_linear import fused_quant as fq

    g = torch.Generator(device=dev).manual_seed(3)
    m, k, i = 4096, 2048, 6144
    x = torch.randn((m, k), generator=g, device=dev).to(torch.bfloat16)
    r = torch.randn((m, k), generator=g, device=dev).to(torch.bfloat16)
    w = (1.0 + 0.1 * torch.randn(k, generator=g, device=dev)).to(torch.bfloat16)
    gu = torch.randn((m, 2 * i), generator=g, device=dev).to(torch.bfloat16)

    def quant(y):
        yf = y.float()
        absmax = yf.abs().amax(-1, keepdim=True)
        inv = torch.where(absmax == 0, torch.zeros_like(absmax), 127.0 / absmax)
        return torch.round(yf * inv).clamp(-128, 127).to(torch.int8), absmax / 127.0

    xf = x.float() + r.float()
    y = ((xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)).to(w.dtype) * w).to(x.dtype)
    q0, s0 = quant(y)
    q, s, _ = fq.add_rmsnorm_quant(x, r, w, 1e-6, True)
    gf, uf = gu[:, :i].float(), gu[:, i:].float()
    a = (gf / (1.0 + torch.exp(-gf))).to(gu.dtype).float()
    q1, s1 = quant((a * uf).to(gu.dtype))
    qs, ss = fq.silu_mul_quant(gu, True, True)
    out = {}
    for name, got, want, sg, sw in (("add_rmsnorm_quant", q, q0, s, s0), ("silu_mul_quant", qs, q1, ss, s1)):
        d = (got.int() - want.int()).abs()
        out[name] = {"differ": int(d.ne(0).sum().item()), "numel": d.numel(),
                     "max_abs": int(d.max().item()),
                     "scale_rel": float(f"{((sg - sw).abs() / sw.clamp_min(1e-30)).max().item():.2g}")}
    return out


# ------------------------------------------------------------------- our arm
def per_shape_timings(cases, graphs, pk):
    from int8_linear.kernel import choose_config

    rows = []
    for (lay, m, bias), g in zip(cases, graphs):
        us = time_graph(g) / COPIES
        k, n = lay["k"], lay["nl"]
        by, ops = alg_bytes(m, k, n, bias), 2 * m * n * k
        t_hbm, t_tc = by / (pk["hbm_gbs"] * 1e3), ops / (pk["int8_tops"] * 1e6)
        rows.append({"layer": lay["name"], "M": m, "K": k, "N": n, "bias": bias, "us": round(us, 3),
                     "bound": "hbm" if t_hbm >= t_tc else "tensor",
                     "roof_frac": round(max(t_hbm, t_tc) / us, 4),
                     "gbs": round(by / us / 1e3, 1), "tops": round(ops / us / 1e6, 1),
                     "tile": choose_config(m, n, k).name})
    return rows


def roofline_of(per_shape, pk):
    """Roofline of the GEMM kernel by class: Σ algorithmic bytes (HBM-bound decode
    shapes) or ops (tensor-bound prefill shapes) over Σ CUDA-event time of the class.
    `traffic` is ncu's DRAM bytes per launch of the class (profiles/gemm_traffic.json)."""
    cls = {"hbm": [0.0, 0.0, 0], "tensor": [0.0, 0.0, 0]}
    for row in per_shape:
        k, n, m = row["K"], row["N"], row["M"]
        amount = alg_bytes(m, k, n, row["bias"]) if row["bound"] == "hbm" else 2 * m * n * k
        cls[row["bound"]][0] += amount
        cls[row["bound"]][1] += row["us"]
        cls[row["bound"]][2] += 1
    tf = ROOT / "profiles" / "gemm_traffic.json"
    traffic = json.loads(tf.read_text()) if tf.exists() else {}
    total = cls["hbm"][1] + cls["tensor"][1]

    def roof(kind):
        amount, us, count = cls[kind]
        if us == 0:
            return None
        if kind == "hbm":
            ach = amount / us / 1e3
            r = {"bound": "hbm", "achieved": round(ach, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                 "frac": round(ach / pk["hbm_gbs"], 4), "traffic": traffic.get("hbm"),
                 "peak_source": pk["source"] + " hbm copy"}
        else:
            ach = amount / us / 1e6
            r = {"bound": "tensor", "achieved": round(ach, 1), "peak": pk["int8_tops"], "unit": "TOPS",
                 "frac": round(ach / pk["int8_tops"], 4), "traffic": traffic.get("tensor"),
                 "peak_source": pk["int8_source"]}
        r["time_share"] = round(us / total, 3)
        r["launches"] = count
        return r

    main = "hbm" if cls["hbm"][1] >= cls["tensor"][1] else "tensor"
    return roof(main), roof("tensor" if main == "hbm" else "hbm")


def timed_sweep(graphs, steps, warmup, world, dev, clocks=None):
    """Device µs per step of replaying every graph once, max over ranks."""
    import torch
    import torch.distributed as dist

    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        for g in graphs:
            g.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ctx = clocks if clocks is not None else _Null()
    with ctx:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("timed_region")   # `ncu --nvtx --nvtx-include timed_region/`
        t0.record(stream)
        for _ in range(steps):
            for g in graphs:
                g.replay()
        t1.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    ms = t0.elapsed_time(t1) / steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


def run_ours(args, world, rank, dev):
    import torch
    import torch.distributed as dist

    from int8_linear import w8a8_mm

    peak = int8_peak_probe(dev)  # every rank on its own GPU; the line reports rank 0's
    pk = peaks(peak["peak"] if peak else None)
    layers, acts = build_operands(args.model, world, rank, dev)
    cases = sweep_cases(layers)
    check = check_sweep(layers, acts, cases)
    graphs = capture_sweep(layers, acts, cases)
    per_shape = per_shape_timings(cases, graphs, pk)
    # L2-warm numbers (the reference's method: the same weight replayed), no-bias cases
    warm = {}
    for lay, m, bias in cases:
        if bias:
            continue
        g = capture(launcher(acts, lay, m, False, [lay["copies"][0]] * COPIES))
        warm[f"{lay['name']}/{m}"] = round(time_graph(g, flush=False) / COPIES, 3)
        del g

    clocks = ClockSampler(dev.index)
    ms = timed_sweep(graphs, args.steps, args.warmup, world, dev, clocks=clocks)
    value_us = ms * 1e3 / COPIES
    roofline, other = roofline_of(per_shape, pk)

    # ------------------------------------------------ all-gather of column shards
    allgather_us = None
    if world > 1:
        tot = 0.0
        for lay, m, bias in cases:
            if bias:
                continue
            local = torch.empty((m, lay["nl"]), dtype=torch.bfloat16, device=dev)
            full = torch.empty((world * m, lay["nl"]), dtype=torch.bfloat16, device=dev)
            for _ in range(3):
                dist.all_gather_into_tensor(full, local)
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(10):
                dist.all_gather_into_tensor(full, local)
            b.record()
            torch.cuda.synchronize()
            tot += a.elapsed_time(b) * 1e3 / 10
        t = torch.tensor([tot], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        allgather_us = round(float(t.item()), 2)

    # ------------------------------------------------ end to end through the public API
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(layers, acts, cases, dev, world, max(1, min(args.steps, 5)))
    del graphs, layers, acts
    torch.cuda.empty_cache()

    # ------------------------------------------------ config 2 (Llama-3-8B), same method
    config2 = None
    if not args.no_config2 and args.model != "llama-3-8b":
        l2, a2 = build_operands("llama-3-8b", world, rank, dev)
        c2 = sweep_cases(l2)
        g2 = capture_sweep(l2, a2, c2)
        config2 = round(timed_sweep(g2, 3, 2, world, dev) * 1e3 / COPIES, 2)
        del g2, l2, a2, c2
        torch.cuda.empty_cache()

    standin = quant = standin_tp = standin_tp_peer = host = ties = None
    if not args.no_standin and world == 1:
        standin = run_standin(dev)
        quant = run_quantisers(dev, pk)
        ties = tie_counts(dev)
        import int8_linear.vllm_patch  # noqa: F401  (registers the custom op)
        from int8_linear import fused_quant as fq_ours
        host = host_cost(w8a8_mm, torch.ops.int8_linear.w8a8_mm, fq_ours, dev)
    if not args.no_standin and world > 1:
        from int8_linear.tp import PeerComm

        standin_tp = run_standin_tp(dev, rank, world)
        comm = PeerComm(device=dev)
        try:
            standin_tp_peer = run_standin_tp(dev, rank, world, comm)
        finally:
            comm.close()

    launches = args.steps * len(cases) * COPIES
    line = {
        "value": round(value_us, 2), "ms_per_step": round(ms, 4), "roofline": roofline,
        "roofline_other": other, "int8_tops_measured": peak, **check, "e2e": e2e,
        "allgather_us_per_sweep": allgather_us, "config2_us_per_sweep": config2,
        "standin_us_per_layer": standin,
        "quantisers_us": ({m: [quant[m]["add_rmsnorm_quant_us"], quant[m]["silu_mul_quant_us"]]
                           for m in QUANT_M_LINE} if quant else None),
        "ties_4096": ({k: v["differ"] for k, v in ties.items()} if ties else None),
        "standin_tp_us_per_layer": standin_tp, "standin_tp_peer_us_per_layer": standin_tp_peer,
        "host_us_per_call": host, "clocks": clocks.summary(), "gpu_launches": launches,
    }
    detail = {"per_shape": per_shape, "l2_warm_us": warm, "quantisers": quant, "ties": ties}
    return line, detail


def host_cost(mm, op, fq, dev) -> dict:
    """The host side of an eager call: µs per call of back-to-back eager calls
    at M=1 (qkv 2048 x 4096), where the host, not the GPU, sets the pace.  The same
    function times both arms (`mm`/`op`/`fq` are the arm's w8a8_mm, custom op and
    fused_quant module)."""
    import torch

    a = torch.randint(-127, 128, (1, 2048), dtype=torch.int8, device=dev)
    w = torch.randint(-127, 128, (4096, 2048), dtype=torch.int8, device=dev)
    sa, sb = torch.rand((1, 1), device=dev), torch.rand((4096, 1), device=dev)
    x = torch.randn((1, 2048), device=dev).to(torch.bfloat16)
    gam = torch.ones(2048, device=dev, dtype=torch.bfloat16)
    gu = torch.randn((1, 12288), device=dev).to(torch.bfloat16)
    out = {}

    def t(name, fn, n=2000, reps=3):
        best = float("inf")
        for _ in range(reps):    # best of `reps` runs: other host activity only adds time
            for _ in range(200):
                fn()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for _ in range(n):
                fn()
            t1 = time.perf_counter()
            torch.cuda.synchronize()
            best = min(best, (t1 - t0) / n)
        out[name] = round(best * 1e6, 2)

    t("w8a8_mm", lambda: mm(a, w.t(), sa, sb, torch.bfloat16))
    t("custom_op_w8a8_mm", lambda: op(a, w.t(), sa, sb, torch.bfloat16, None))
    t("add_rmsnorm_quant", lambda: fq.add_rmsnorm_quant(x, x, gam, 1e-6, True))
    t("silu_mul_quant", lambda: fq.silu_mul_quant(gu, True, True))
    return out


E2E_GROUPS = 12


def run_e2e(layers, acts, cases, dev, world, passes):
    """The sweep through w8a8_mm with host buffers: every step copies each case's int8
    activations and scales from pinned memory to the GPU, runs the GEMM, and copies its
    output back into pinned memory.  The cases go in E2E_GROUPS groups of consecutive
    cases; a group's inputs are packed in one pinned buffer (one H2D copy) and its
    outputs in one device buffer (one D2H copy), so PCIe moves large copies instead of
    288 small ones.  The two directions run on their own streams and overlap each other
    and the GEMMs, ordered by events: a group's GEMMs wait for its H2D and for the D2H of
    its output buffer in the previous pass; its D2H waits for its GEMMs; its next H2D
    waits for its GEMMs."""
    import torch
    import torch.distributed as dist

    from int8_linear import w8a8_mm

    def up(x, a=256):
        return -(-x // a) * a

    per = -(-len(cases) // E2E_GROUPS)
    groups = []
    h2d = d2h = 0
    for g0 in range(0, len(cases), per):
        items, in_off, out_off = [], 0, 0
        for lay, m, bias in cases[g0:g0 + per]:
            a_q, a_s = acts[(m, lay["k"])]
            qa, sa_off = in_off, in_off + up(a_q.numel())
            in_off = sa_off + up(a_s.numel() * 4)
            items.append((lay, m, bias, a_q, a_s, qa, sa_off, out_off))
            out_off += up(m * lay["nl"] * 2)
        host_in = torch.empty(in_off, dtype=torch.uint8).pin_memory()
        for lay, m, bias, a_q, a_s, qa, sa_off, _ in items:
            host_in[qa:qa + a_q.numel()].copy_(a_q.cpu().reshape(-1).view(torch.uint8))
            host_in[sa_off:sa_off + a_s.numel() * 4].copy_(a_s.cpu().reshape(-1).view(torch.uint8))
        dev_in = torch.empty(in_off, dtype=torch.uint8, device=dev)
        dev_out = torch.empty(out_off, dtype=torch.uint8, device=dev)
        host_out = torch.empty(out_off, dtype=torch.uint8).pin_memory()
        views = []
        for lay, m, bias, a_q, a_s, qa, sa_off, oo in items:
            k, n = lay["k"], lay["nl"]
            views.append((lay, bias, dev_in[qa:qa + m * k].view(torch.int8).view(m, k),
                          dev_in[sa_off:sa_off + m * 4].view(torch.float32).view(m, 1),
                          dev_out[oo:oo + m * n * 2].view(torch.bfloat16).view(m, n)))
        groups.append((host_in, dev_in, dev_out, host_out, views))
        h2d += in_off
        d2h += out_off

    turn = {}
    comp = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    gemms_done, copied_out = {}, {}

    def one_pass():
        for gi, (host_in, dev_in, dev_out, host_out, views) in enumerate(groups):
            with torch.cuda.stream(s_in):
                if gi in gemms_done:
                    s_in.wait_event(gemms_done[gi])
                dev_in.copy_(host_in, non_blocking=True)
                landed = torch.cuda.Event()
                landed.record(s_in)
            comp.wait_event(landed)
            if gi in copied_out:
                comp.wait_event(copied_out[gi])
            for lay, bias, da, ds, do in views:
                i = turn[lay["name"]] = (turn.get(lay["name"], -1) + 1) % len(lay["copies"])
                wq, ws = lay["copies"][i]
                w8a8_mm(da, wq.t(), ds, ws, torch.bfloat16, lay["bias"] if bias else None, out=do)
            ev = gemms_done[gi] = torch.cuda.Event()
            ev.record(comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev)
                host_out.copy_(dev_out, non_blocking=True)
                done_out = copied_out[gi] = torch.cuda.Event()
                done_out.record(s_out)

    one_pass()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    s_in.wait_stream(comp)
    for _ in range(passes):
        one_pass()
    comp.wait_stream(s_out)
    b.record()
    torch.cuda.synchronize()
    us = a.elapsed_time(b) * 1e3 / passes
    if world > 1:
        t = torch.tensor([us], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        us = float(t.item())
    return {"value": round(us, 2), "unit": "us", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "passes": passes,
            "note": f"eager sweep through w8a8_mm; {len(groups)} packed H2D + D2H copies per pass, "
                    "overlapped on their own streams"}


def run_standin_tp(dev, rank, world, comm=None):
    """BASELINE config 4 under tensor parallelism: the stand-in decoder split over the
    ranks (int8_linear/tp.py), µs per layer, max over ranks.  With `comm` (a PeerComm)
    the exchanges run in the library's NVLink kernels, else in NCCL collectives."""
    import torch
    import torch.distributed as dist

    from int8_linear.standin import LAYERS, TPStandinDecoder

    out = {}
    for m in STANDIN_BATCHES:
        s = TPStandinDecoder(m, rank, world, device=dev, comm=comm)
        g = s.capture()
        dist.barrier()
        us = statistics.median([time_graph(g, windows=5) for _ in range(3)]) / LAYERS
        t = torch.tensor([us], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        out[str(m)] = round(float(t.item()), 2)
        torch.cuda.synchronize()
        dist.barrier()
        del g, s
        torch.cuda.empty_cache()
    return out


def run_quantisers(dev, pk):
    """the fused quantisers, µs per call (graph of 50 calls) and the
    fraction of HBM bandwidth their algorithmic bytes reach.  Timed with the run's
    programmatic-dependent-launch setting and, as `*_no_pdl`, without it: 50 identical
    calls back to back are not what PDL is for (each call's CTAs start early beside
    the previous call's on the same SMs); in a decode chain PDL overlaps each kernel
    with the GEMM next to it."""
    import torch

    from int8_linear import _native
    from int8_linear import fused_quant as fq

    out = {}
    pdl = _native.pdl_enabled()
    g = torch.Generator(device=dev).manual_seed(3)
    gamma = (1.0 + 0.1 * torch.randn(2048, generator=g, device=dev)).to(torch.bfloat16)
    for m in QUANT_M:
        x = torch.randn((m, 2048), generator=g, device=dev).to(torch.bfloat16)
        r = torch.randn((m, 2048), generator=g, device=dev).to(torch.bfloat16)
        gu = torch.randn((m, 12288), generator=g, device=dev).to(torch.bfloat16)
        t_norm = time_graph(capture(lambda: [fq.add_rmsnorm_quant(x, r, gamma, 1e-6) for _ in range(50)])) / 50
        t_silu = time_graph(capture(lambda: [fq.silu_mul_quant(gu, True, True) for _ in range(50)])) / 50
        b_norm = m * (2048 * 7 + 4) + 2 * 2048
        b_silu = m * (6144 * 5 + 4)
        _native.set_pdl(False)
        t_norm0 = time_graph(capture(lambda: [fq.add_rmsnorm_quant(x, r, gamma, 1e-6) for _ in range(50)])) / 50
        t_silu0 = time_graph(capture(lambda: [fq.silu_mul_quant(gu, True, True) for _ in range(50)])) / 50
        _native.set_pdl(pdl)
        out[str(m)] = {"add_rmsnorm_quant_us": round(t_norm, 2),
                       "add_rmsnorm_quant_hbm_frac": round(b_norm / t_norm / 1e3 / pk["hbm_gbs"], 3),
                       "silu_mul_quant_us": round(t_silu, 2),
                       "silu_mul_quant_hbm_frac": round(b_silu / t_silu / 1e3 / pk["hbm_gbs"], 3),
                       "add_rmsnorm_quant_us_no_pdl": round(t_norm0, 2),
                       "silu_mul_quant_us_no_pdl": round(t_silu0, 2)}
    return out


def run_standin(dev):
    """28-layer stand-in decode step, one CUDA graph, µs per layer."""
    import torch

    from int8_linear.standin import LAYERS, StandinDecoder

    out = {}
    for m in STANDIN_BATCHES:
        s = StandinDecoder(m, device=dev)
        g = s.capture()
        ts = []
        for _ in range(3):
            ts.append(time_graph(g, windows=5))
        out[str(m)] = round(statistics.median(ts) / LAYERS, 2)
        del g, s
        torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------------- reference arm
def cpu_operands(model, seed=0):
    """The sweep's int8 operands on the CPU, generated as config 0 (bf16 N(0,1)
    activations, N(0,0.02) weights, per-row quantisation; bf16 N(0,0.01) bias): one weight
    per layer and one activation per (M, K)."""
    import torch

    g = torch.Generator().manual_seed(seed)
    layers = []
    for name, k, n in layers_for(model):
        wq, ws = quant_rows_t((torch.randn((n, k), generator=g) * 0.02).to(torch.bfloat16))
        bias = (torch.randn((n,), generator=g) * 0.01).to(torch.bfloat16)
        layers.append((name, k, n, wq, ws, bias))
    acts = {(m, k): quant_rows_t(torch.randn((m, k), generator=g).to(torch.bfloat16))
            for k in sorted({lay[1] for lay in layers}) for m in M_SWEEP}
    return layers, acts


def cpu_sweep_pass(layers, acts) -> float:
    """One pass of the whole sweep (every layer, M and bias; full M x N, no sampling)
    through the reference's CPU float64 layer; returns seconds."""
    from oracle.gemm import layer_f64_torch

    t0 = time.perf_counter()
    for bias in (False, True):
        for _, k, _, wq, ws, b in layers:
            for m in M_SWEEP:
                a_q, a_s = acts[(m, k)]
                layer_f64_torch(a_q, a_s, wq, ws, b if bias else None)
    return time.perf_counter() - t0


def cpu_baseline(model, passes: int, warmup: int = 1) -> dict:
    import torch

    torch.set_num_threads(os.cpu_count() or 1)
    layers, acts = cpu_operands(model)
    for _ in range(warmup):
        cpu_sweep_pass(layers, acts)
    ts = [cpu_sweep_pass(layers, acts) for _ in range(passes)]
    v = statistics.median(ts) * 1e6
    return {"value": round(v, 1), "unit": "us", "cores": torch.get_num_threads(), "kind": "port",
            "cpu": cpu_model(),
            "sample": f"the whole 96-GEMM sweep (every M, N, bias; no sampling) through the reference's "
                      f"float64 torch layer (bench/bench_linear.py:164-165), median of {passes} passes"}


def run_reference(args, world, rank):
    if rank != 0:
        return None
    import torch

    torch.set_num_threads(os.cpu_count() or 1)
    layers, acts = cpu_operands(args.model)
    for _ in range(args.warmup):
        cpu_sweep_pass(layers, acts)
    t0 = time.perf_counter()
    vals = [cpu_sweep_pass(layers, acts) for _ in range(args.steps)]
    wall = time.perf_counter() - t0
    v = statistics.median(vals) * 1e6
    base = {"value": round(v, 1), "unit": "us", "cores": torch.get_num_threads(), "kind": "port",
            "cpu": cpu_model(),
            "sample": "each step: the whole 96-GEMM sweep (every M, N, bias; no sampling) through the "
                      "reference's float64 torch layer (bench/bench_linear.py:164-165); value = median step"}
    return {
        "value": round(v, 1), "ms_per_step": round(wall * 1e3 / args.steps, 2),
        "cpu_baseline": base,
        "e2e": {"value": round(v, 1), "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ------------------------------------------------------------------- reference Triton arm
REF_INSTALL = ROOT / "baseline" / "_ref"


def run_reference_triton_child(args):
    """In a process whose only int8_linear is the installed reference (baseline/_ref):
    its Triton w8a8_mm over the same sweep (L2-cold, same timing) and its stand-in
    (bench/fuse_quant.py Stack.fused structure, vLLM's scaled_int8_quant where the
    reference uses it, else the same per-token quantiser in torch)."""
    import torch

    import int8_linear as ref
    from int8_linear import fused_quant as rfq
    from int8_linear.kernel import w8a8_mm as ref_mm

    assert str(REF_INSTALL) in ref.__file__, ref.__file__
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(1234)
    per = {}
    for name, k, n in layers_for(args.model):
        ws = [quant_rows_t((torch.randn((n, k), generator=g, device=dev) * 0.02).to(torch.bfloat16))
              for _ in range(pool_size(n * k))]
        w0 = 0
        bias = (torch.randn(n, generator=g, device=dev) * 0.01).to(torch.bfloat16)
        for m in M_SWEEP:
            a_q, a_s = quant_rows_t(torch.randn((m, k), generator=g, device=dev).to(torch.bfloat16))
            for b in (None, bias):    # the same 96 cases as our arm: with and without bias
                window = ws[w0:w0 + COPIES]
                w0 = (w0 + COPIES) % len(ws)

                def fn(b=b, window=window):
                    for wq, wsc in window:
                        ref_mm(a_q, wq.t(), a_s, wsc, torch.bfloat16, b)
                key = f"{name}/{m}" + ("" if b is None else "/bias")
                per[key] = round(time_graph(capture(fn)) / COPIES, 3)
        del ws
    total = sum(per.values())
    try:
        from vllm import _custom_ops as ops

        def q8(x):
            q, s_, _ = ops.scaled_int8_quant(x)
            return q, s_
        q8(torch.randn((2, 2048), device=dev).to(torch.bfloat16))
        qsrc = "vllm scaled_int8_quant"
    except Exception as e:  # noqa: BLE001
        qsrc = f"torch per-token quantiser ({type(e).__name__} loading vLLM ops)"

        def q8(x):
            xf = x.float()
            am = xf.abs().amax(-1, keepdim=True)
            inv = torch.where(am == 0, torch.zeros_like(am), 127.0 / am)
            return torch.round(xf * inv).clamp(-128, 127).to(torch.int8), am / 127.0
    # BASELINE config 3 on the reference's Triton quantisers (same method as our arm:
    # graph of 50 calls, µs per call)
    quant = {}
    for m in QUANT_M:
        gq = torch.Generator(device=dev).manual_seed(3)
        xq = torch.randn((m, 2048), generator=gq, device=dev).to(torch.bfloat16)
        rq = torch.randn((m, 2048), generator=gq, device=dev).to(torch.bfloat16)
        gam = (1 + 0.1 * torch.randn(2048, generator=gq, device=dev)).to(torch.bfloat16)
        guq = torch.randn((m, 12288), generator=gq, device=dev).to(torch.bfloat16)
        t_norm = time_graph(capture(lambda: [rfq.add_rmsnorm_quant(xq, rq, gam, 1e-6, True) for _ in range(50)])) / 50
        t_silu = time_graph(capture(lambda: [rfq.silu_mul_quant(guq, True, True) for _ in range(50)])) / 50
        quant[str(m)] = {"add_rmsnorm_quant_us": round(t_norm, 2), "silu_mul_quant_us": round(t_silu, 2)}
    standin = {}
    for m in STANDIN_BATCHES:
        gg = torch.Generator(device=dev).manual_seed(0)
        x = torch.randn((m, 2048), generator=gg, device=dev).to(torch.bfloat16)
        w = torch.ones(2048, device=dev, dtype=torch.bfloat16)
        layers = []
        for _ in range(28):
            layer = {}
            for nm, (k, n) in {"qkv": (2048, 4096), "o": (2048, 2048), "gu": (2048, 12288),
                               "dn": (6144, 2048)}.items():
                wq = torch.randint(-127, 128, (n, k), generator=gg, device=dev, dtype=torch.int8)
                layer[nm] = (wq.t(), torch.rand((n, 1), generator=gg, device=dev) * 1e-3 + 1e-4)
            layers.append(layer)

        def step():
            res = x
            q, s_, _ = rfq.add_rmsnorm_quant(x, None, w, 1e-6, True)
            h = None
            for i, L in enumerate(layers):
                if i:
                    q, s_, res = rfq.add_rmsnorm_quant(h, res, w, 1e-6, True)
                a = ref_mm(q, L["qkv"][0], s_, L["qkv"][1], torch.bfloat16)[:, :2048].contiguous()
                q, s_ = q8(a)
                h = ref_mm(q, L["o"][0], s_, L["o"][1], torch.bfloat16)
                q, s_, res = rfq.add_rmsnorm_quant(h, res, w, 1e-6, True)
                gu = ref_mm(q, L["gu"][0], s_, L["gu"][1], torch.bfloat16)
                q, s_ = rfq.silu_mul_quant(gu, True, True)
                h = ref_mm(q, L["dn"][0], s_, L["dn"][1], torch.bfloat16)
            return h
        standin[str(m)] = round(statistics.median([time_graph(capture(step)) for _ in range(3)]) / 28, 2)
        del layers
        torch.cuda.empty_cache()
    import int8_linear.vllm_patch  # noqa: F401  (registers the reference's custom op)
    host = host_cost(ref_mm, torch.ops.int8_linear.w8a8_mm, rfq, dev)
    print(json.dumps({"value": round(total, 2), "per_shape_us": per, "standin_us_per_layer": standin,
                      "quantisers": quant, "host_us_per_call": host,
                      "standin_o_proj_quantiser": qsrc, "triton": __import__("triton").__version__}))


def run_reference_triton(args, rank):
    """The reference's own Triton kernels on this GPU (not the CPU reference arm):
    a child process with PYTHONPATH set to the installed reference."""
    if rank != 0:
        return None
    if not (REF_INSTALL / "int8_linear").exists():
        return {"unavailable": "the reference is not installed under baseline/_ref"}
    env = dict(os.environ, PYTHONPATH=str(REF_INSTALL))
    cmd = [sys.executable, str(ROOT / "bench.py"), "--impl", "reference-triton-child",
           "--model", args.model]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=1800)
    if r.returncode != 0:
        return {"unavailable": "reference Triton run failed: " + (r.stderr.strip().splitlines() or ["?"])[-1]}
    return json.loads(r.stdout.strip().splitlines()[-1])


# ------------------------------------------------------------------- profiling cases
def run_case(args) -> None:
    """Small, self-contained workloads for profiling one kernel (e.g. under ncu): each runs
    a few launches (`--iters`) after the first, so `ncu -s <skip> -c <count>` can pick
    steady-state launches, and keeps the device footprint small.

        --case gemm --shape M,N,K [--config bm,bn[,split[,cluster[,swap]]]]   one GEMM, 2 weights
        --case sweep [--model M]                                      every (layer, M) once
        --case quant --shape M --kind norm|silu|plain                 one quantiser
        --case dequant --shape M,N                                    int32 product -> bf16
        --case standin --shape B                                      stand-in step replays
    """
    import torch

    from int8_linear import fused_quant as fq
    from int8_linear import set_pdl, w8a8_mm
    from int8_linear.kernel import Config

    set_pdl(not args.no_pdl)
    g = torch.Generator(device="cuda").manual_seed(0)

    def ints(shape):
        return torch.randint(-127, 128, shape, dtype=torch.int8, device="cuda", generator=g)

    if args.case == "gemm":
        m, n, k = (int(v) for v in args.shape.split(","))
        cfg = None
        if args.config:
            f = [int(v) for v in args.config.split(",")]
            cfg = Config(f[0], f[1], split=f[2] if len(f) > 2 else 0, cluster=f[3] if len(f) > 3 else 0,
                         swap_ab=bool(f[4]) if len(f) > 4 else None)
        a, ws = ints((m, k)), [ints((n, k)) for _ in range(2)]
        sa = torch.rand((m, 1), device="cuda", generator=g) * 1e-2 + 1e-3
        sb = torch.rand((n, 1), device="cuda", generator=g) * 1e-3 + 1e-4
        for i in range(args.iters):
            w8a8_mm(a, ws[i % 2].t(), sa, sb, torch.bfloat16, config=cfg)
    elif args.case == "sweep":
        for _, k, n in layers_for(args.model):
            w = ints((n, k))
            sb = torch.rand((n, 1), device="cuda", generator=g) * 1e-3 + 1e-4
            for m in M_SWEEP:
                sa = torch.rand((m, 1), device="cuda", generator=g) * 1e-2 + 1e-3
                w8a8_mm(ints((m, k)), w.t(), sa, sb, torch.bfloat16)
            torch.cuda.synchronize()
    elif args.case == "quant":
        m = int(args.shape)
        x = torch.randn((m, 2048), device="cuda", generator=g).to(torch.bfloat16)
        r = torch.randn((m, 2048), device="cuda", generator=g).to(torch.bfloat16)
        gamma = (1 + 0.1 * torch.randn(2048, device="cuda", generator=g)).to(torch.bfloat16)
        gu = torch.randn((m, 12288), device="cuda", generator=g).to(torch.bfloat16)
        for _ in range(args.iters):
            if args.kind == "norm":
                fq.add_rmsnorm_quant(x, r, gamma, 1e-6)
            elif args.kind == "silu":
                fq.silu_mul_quant(gu, True, True)
            else:
                fq.per_token_quant(x)
    elif args.case == "dequant":
        from int8_linear.kernel import dequant_i32

        m, n = (int(v) for v in args.shape.split(","))
        acc = torch.randint(-(1 << 20), 1 << 20, (m, n), dtype=torch.int32, device="cuda", generator=g)
        sa = torch.rand((m, 1), device="cuda", generator=g) * 1e-2 + 1e-3
        sb = torch.rand((n, 1), device="cuda", generator=g) * 1e-3 + 1e-4
        for _ in range(args.iters):
            dequant_i32(acc, sa, sb, torch.bfloat16)
    else:
        from int8_linear.standin import StandinDecoder

        s = StandinDecoder(int(args.shape or 1))
        gr = s.capture()
        for _ in range(args.iters):
            gr.replay()
    torch.cuda.synchronize()
    print(json.dumps({"case": args.case, "shape": args.shape, "iters": args.iters}), flush=True)


# ------------------------------------------------------------------- main
def short_line(line: dict) -> str:
    """The final JSON line, dropping optional tables (largest first) if it would exceed
    LINE_LIMIT bytes."""
    drop = ["int8_tops_measured", "host_us_per_call", "standin_tp_peer_us_per_layer",
            "standin_tp_us_per_layer", "quantisers_us"]
    s = json.dumps(line)
    for key in drop:
        if len(s.encode()) <= LINE_LIMIT:
            break
        line.pop(key, None)
        s = json.dumps(line)
    return s


def detail_path(args, world) -> Path:
    if args.detail:
        return Path(args.detail)
    return ROOT / "gpurun_out" / f"bench_detail_n{world}.json"


def main():
    args = parse()
    if args.case:
        run_case(args)
        return
    if args.impl == "reference-triton-child":
        # Only the installed reference may provide int8_linear in this process.
        sys.path[:] = [str(REF_INSTALL)] + [p for p in sys.path if Path(p or ".").resolve() != ROOT]
        run_reference_triton_child(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    base = {"metric": METRIC, "unit": "us", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "data": "synthetic",
            "config": {"workload": f"per-layer sweep, {args.model} (BASELINE config "
                                   f"{1 if args.model.startswith('qwen') else 2})",
                       "layers": [f"{nm} K={k} N={n}" for nm, k, n in layers_for(args.model)],
                       "M": M_SWEEP, "bias": [False, True],
                       "l2": (f"cold: {COPIES} launches per case on distinct weight copies from a pool "
                              "of at least 2x L2 per layer"),
                       "parallelism": f"column-parallel N/{world}" if world > 1 else "single GPU",
                       "pdl": not args.no_pdl}}
    if args.impl == "reference-triton":
        res = run_reference_triton(args, rank)
        if rank == 0:
            print(json.dumps(dict(base, impl="reference-triton", dtype="i8", **res)), flush=True)
        return
    if args.impl == "reference":
        res = run_reference(args, world, rank)
        if rank == 0:
            line = dict(base, impl="reference", dtype="f64", **res)
            print(json.dumps(line), flush=True)
        return

    import torch
    import torch.distributed as dist

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    from int8_linear import set_pdl

    set_pdl(not args.no_pdl)  # inference weights are read-only: let kernels overlap
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    line, detail = run_ours(args, world, rank, dev)
    cpu = None
    if world == 1 and rank == 0:
        cpu = cpu_baseline(args.model, passes=3)
    if rank == 0:
        dpath = detail_path(args, world)
        dpath.parent.mkdir(parents=True, exist_ok=True)
        full = {**base, "dtype": "i8", "cpu_baseline": cpu, **line, **detail}
        dpath.write_text(json.dumps(full, indent=1) + "\n")
        out = dict(base, dtype="i8", cpu_baseline=cpu, **line)
        out["detail"] = os.path.relpath(dpath, ROOT)
        s = short_line(out)
        print(s, flush=True)
        if args.out:
            Path(args.out).write_text(s + "\n")
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
