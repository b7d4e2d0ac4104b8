"""A 28-layer Qwen3-1.7B-shaped decoder with attention left out, on this library's kernels.

The reference measures its fused path on this stand-in (bench/fuse_quant.py:184-240,
class Stack, method fused): every layer has its own seeded int8 weights, and one decode
step runs, per layer,

    add_rmsnorm_quant -> qkv GEMM -> (first 2048 columns) per-token quant -> o_proj GEMM
    -> add_rmsnorm_quant -> gate_up GEMM -> silu_mul_quant -> down GEMM

captured as one CUDA graph.  Here the qkv slice is quantised in place (the quantiser
reads rows with a stride), where the reference copies it with .contiguous() and then
calls vLLM's scaled_int8_quant; the values are the same.

With `fuse` (the default), every linear whose tiling is a CUDA-core tile (decode batches
of a few tokens) takes its quantiser into the GEMM's prologue: add_rmsnorm_quant ->
qkv_proj becomes rmsnorm_w8a8_mm, quant -> o_proj w8a8_mm_quant_act, add_rmsnorm_quant ->
gate_up_proj rmsnorm_w8a8_mm and silu_mul_quant -> down_proj silu_mul_w8a8_mm, each one
launch with the same bits as the two it replaces (a batch the fused kernel declines runs
the two steps).  With fuse_o_proj, o_proj's quantiser also runs inside tensor-core tilings
that have direct activation loads (w8a8_mm_quant_act); off by default, as those tilings
were measured slower on B200 than the quantiser followed by the tuned tiling.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from int8_linear.fused_quant import add_rmsnorm_quant, per_token_quant, silu_mul_quant
from int8_linear import kernel
from int8_linear.kernel import (Config, choose_config, rmsnorm_w8a8_mm, silu_mul_w8a8_mm, w8a8_mm,
                                w8a8_mm_quant_act)

HIDDEN, INTER, EPS, LAYERS = 2048, 6144, 1e-6, 28
# Linears whose quantiser goes into the GEMM prologue, per decode batch, when `fuse` is
# True: where it was measured faster in the 28-layer step on B200 (every CTA re-reads the
# batch's bf16 activation, so the fusion pays only while that is small).
# Per linear, µs per layer against no fusion (28 layers, L2-cold): batch 1 o_proj -1.5,
# gate_up -0.4, qkv +0.4, down +1.7; batch 2 o_proj -0.2, the others +1 to +3; from batch 4
# every fusion slower.
FUSE_DEFAULT: dict[int, tuple[str, ...]] = {1: ("o_proj", "gate_up_proj"), 2: ("o_proj",)}
# (K, N) of each linear, as vLLM runs Qwen3-1.7B (merged qkv and gate_up).
SHAPES = {"qkv_proj": (2048, 4096), "o_proj": (2048, 2048),
          "gate_up_proj": (2048, 12288), "down_proj": (6144, 2048)}


@dataclass
class Linear:
    w_t: torch.Tensor    # [K, N] view of the [N, K] int8 weight (K-contiguous)
    scale: torch.Tensor  # [N, 1] float32


def make_layers(layers: int = LAYERS, seed: int = 0, device="cuda", shapes=SHAPES,
                generator: torch.Generator | None = None) -> list[dict[str, Linear]]:
    """Per-layer int8 weights randint(-127, 128) and scales rand*1e-3 + 1e-4, drawn from one
    seeded generator in layer order (bench/fuse_quant.py:194-199)."""
    g = generator or torch.Generator(device=device).manual_seed(seed)
    out = []
    for _ in range(layers):
        layer = {}
        for name, (k, n) in shapes.items():
            wq = torch.randint(-127, 128, (n, k), generator=g, device=device, dtype=torch.int8)
            layer[name] = Linear(wq.t(), torch.rand((n, 1), generator=g, device=device) * 1e-3 + 1e-4)
        out.append(layer)
    return out


class StandinDecoder:
    """The reference's fused stand-in step for a decode batch of m tokens.

    `configs` maps a linear's name (a key of SHAPES) to the tiling its GEMMs use in every
    layer; linears not named use the library's choice (choose_config).  It may be changed
    between captures (the in-situ tuner does)."""

    def __init__(self, m: int, layers: int = LAYERS, seed: int = 0, device="cuda",
                 norm_weight: torch.Tensor | None = None, configs: dict[str, Config] | None = None,
                 fuse_o_proj: bool = False, fuse: bool | set[str] = True):
        g = torch.Generator(device=device).manual_seed(seed)
        self.x = torch.randn((m, HIDDEN), generator=g, device=device).to(torch.bfloat16)
        self.w = (norm_weight if norm_weight is not None
                  else torch.ones(HIDDEN, device=device, dtype=torch.bfloat16))
        self.layers = make_layers(layers, device=device, generator=g)
        self.configs: dict[str, Config] = dict(configs or {})
        self.fuse_o_proj = fuse_o_proj
        # True: the library's choice per linear (FUSE_DEFAULT); False: none; or a set of
        # the linears (keys of SHAPES) whose quantiser goes into the GEMM prologue.
        self.fuse = fuse
        self.graph: torch.cuda.CUDAGraph | None = None
        self.out: torch.Tensor | None = None

    def _cuda_core(self, name: str) -> bool:
        """Whether the linear `name` runs on a CUDA-core tile at this batch."""
        k, n = SHAPES[name]
        cfg = self.configs.get(name) or choose_config(self.x.shape[0], n, k)
        return cfg.split == 5

    def fused(self, name: str) -> bool:
        """Whether the linear `name` takes its quantiser into its GEMM's prologue."""
        if self.fuse is True:
            return name in FUSE_DEFAULT.get(self.x.shape[0], ())
        return bool(self.fuse) and name in self.fuse

    def step(self, record: list | None = None) -> torch.Tensor:
        """One decode step.  With `record` (a list), every op appends (layer, op name,
        inputs, outputs), so a test can check each op on its own inputs."""
        if self.fuse:
            return self._step_fused(record)
        cfg = self.configs.get

        def rec(i, name, ins, outs):
            if record is not None:
                record.append((i, name, ins, outs))
            return outs

        res = self.x
        q, s, _ = rec(-1, "norm", (self.x, None, self.w), add_rmsnorm_quant(self.x, None, self.w, EPS))
        h = None
        for i, layer in enumerate(self.layers):
            if i:
                q, s, res = rec(i, "norm", (h, res, self.w), add_rmsnorm_quant(h, res, self.w, EPS))
            lin = layer["qkv_proj"]
            qkv = rec(i, "qkv_proj", (q, s, lin),
                      w8a8_mm(q, lin.w_t, s, lin.scale, torch.bfloat16, config=cfg("qkv_proj")))
            lin = layer["o_proj"]
            if self.fuse_o_proj:
                h = rec(i, "o_proj_quant_act", (qkv[:, :HIDDEN], lin),
                        w8a8_mm_quant_act(qkv[:, :HIDDEN], lin.w_t, lin.scale, torch.bfloat16,
                                          config=cfg("o_proj")))
            else:
                q, s = rec(i, "quant", (qkv[:, :HIDDEN],), per_token_quant(qkv[:, :HIDDEN]))
                h = rec(i, "o_proj", (q, s, lin),
                        w8a8_mm(q, lin.w_t, s, lin.scale, torch.bfloat16, config=cfg("o_proj")))
            q, s, res = rec(i, "post_norm", (h, res, self.w), add_rmsnorm_quant(h, res, self.w, EPS))
            lin = layer["gate_up_proj"]
            gu = rec(i, "gate_up_proj", (q, s, lin),
                     w8a8_mm(q, lin.w_t, s, lin.scale, torch.bfloat16, config=cfg("gate_up_proj")))
            q, s = rec(i, "silu_mul_quant", (gu,), silu_mul_quant(gu))
            lin = layer["down_proj"]
            h = rec(i, "down_proj", (q, s, lin),
                    w8a8_mm(q, lin.w_t, s, lin.scale, torch.bfloat16, config=cfg("down_proj")))
        return h

    def _step_fused(self, record: list | None) -> torch.Tensor:
        """The step with each quantiser in the prologue of the GEMM it feeds, wherever that
        GEMM runs on a CUDA-core tile (the same bits as step without fuse)."""
        cfg = self.configs.get

        def rec(i, name, ins, outs):
            if record is not None:
                record.append((i, name, ins, outs))
            return outs

        def norm_mm(i, name, x_in, r_in, lin):
            if self.fused(name):
                return rec(i, "norm_" + name, (x_in, r_in, self.w, lin),
                           rmsnorm_w8a8_mm(x_in, r_in, self.w, EPS, lin.w_t, lin.scale,
                                           config=cfg(name)))
            q, s, rout = rec(i, "norm" if name == "qkv_proj" else "post_norm", (x_in, r_in, self.w),
                             add_rmsnorm_quant(x_in, r_in, self.w, EPS))
            return rec(i, name, (q, s, lin),
                       w8a8_mm(q, lin.w_t, s, lin.scale, torch.bfloat16, config=cfg(name))), rout

        res = self.x
        h = None
        for i, layer in enumerate(self.layers):
            x_in, r_in = (self.x, None) if i == 0 else (h, res)
            qkv, rout = norm_mm(i, "qkv_proj", x_in, r_in, layer["qkv_proj"])
            if i:
                res = rout
            lin = layer["o_proj"]
            if self.fused("o_proj") or self.fuse_o_proj:
                h = rec(i, "quant_o_proj", (qkv[:, :HIDDEN], lin),
                        w8a8_mm_quant_act(qkv[:, :HIDDEN], lin.w_t, lin.scale, torch.bfloat16,
                                          config=cfg("o_proj")))
            else:
                q, s = rec(i, "quant", (qkv[:, :HIDDEN],), per_token_quant(qkv[:, :HIDDEN]))
                h = rec(i, "o_proj", (q, s, lin),
                        w8a8_mm(q, lin.w_t, s, lin.scale, torch.bfloat16, config=cfg("o_proj")))
            gu, res = norm_mm(i, "gate_up_proj", h, res, layer["gate_up_proj"])
            lin = layer["down_proj"]
            if self.fused("down_proj"):
                h = rec(i, "silu_down_proj", (gu, lin),
                        silu_mul_w8a8_mm(gu, lin.w_t, lin.scale, config=cfg("down_proj")))
            else:
                q, s = rec(i, "silu_mul_quant", (gu,), silu_mul_quant(gu))
                h = rec(i, "down_proj", (q, s, lin),
                        w8a8_mm(q, lin.w_t, s, lin.scale, torch.bfloat16, config=cfg("down_proj")))
        return h

    def capture(self) -> torch.cuda.CUDAGraph:
        """Capture one step into a CUDA graph (after a warm-up call on a side stream),
        replacing any earlier capture."""
        self.graph = None
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            self.step()
        torch.cuda.current_stream().wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = self.step()
        return self.graph

    def o_proj_fused(self) -> bool:
        """Whether o_proj's input quantisation runs inside its GEMM at this batch."""
        if self.fused("o_proj") and self._cuda_core("o_proj"):
            return True
        if not self.fuse_o_proj:
            return False
        m = self.x.shape[0]
        k, n = SHAPES["o_proj"]
        if self.configs.get("o_proj") is not None:
            return kernel.fused_act_config(self.configs["o_proj"]) is not None
        return kernel._fused_chosen.get((self.x.get_device(), m, n, k)) is not None

    @property
    def launches_per_step(self) -> int:
        """Kernels one step launches (counted by recording an eager step)."""
        rec: list = []
        self.step(record=rec)
        two = {"norm_qkv_proj", "norm_gate_up_proj", "silu_down_proj", "quant_o_proj"}
        count = 0
        for _, name, ins, _ in rec:
            if name in two and not self._fused_call(name, ins):
                count += 2
            else:
                count += 1
        return count

    def _fused_call(self, name: str, ins) -> bool:
        """Whether a fused record ran as one kernel (its GEMM on a CUDA-core tile whose
        prologue takes this quantiser)."""
        lin_name = {"norm_qkv_proj": "qkv_proj", "norm_gate_up_proj": "gate_up_proj",
                    "silu_down_proj": "down_proj", "quant_o_proj": "o_proj"}[name]
        if not self._cuda_core(lin_name):
            return name == "quant_o_proj" and self.o_proj_fused()
        if name == "quant_o_proj":
            return True
        m = self.x.shape[0]
        k = SHAPES[lin_name][0]
        vecs = k // 8
        nv = next(v for v in (1, 2, 3, 4, 6, 8, 12, 16) if -(-vecs // v) <= 256)
        mt = next(t for t in kernel.GEMV_TOKENS if t >= m)
        return nv <= 3 and mt * nv <= 8

    def weight_bytes(self) -> int:
        return sum(lin.w_t.numel() + lin.scale.numel() * 4 for layer in self.layers
                   for lin in layer.values())


class TPStandinDecoder:
    """The stand-in decoder split over `world` GPUs, Megatron-style (int8_linear/tp.py):
    qkv and gate_up column-parallel (q, k, v and gate, up sharded separately), o_proj and
    down row-parallel with an exact int32 all-reduce, the row-split activations quantised
    with the global per-token absmax.  Built from the same seeded weights as
    StandinDecoder, so every rank's output equals the one-GPU output bit for bit.  With
    `comm` (a tp.PeerComm) the exchanges run in this library's NVLink kernels, else in
    NCCL collectives."""

    def __init__(self, m: int, rank: int, world: int, group=None, layers: int = LAYERS,
                 seed: int = 0, device="cuda", comm=None):
        from int8_linear import tp

        full = StandinDecoder(m, layers=layers, seed=seed, device=device)
        self.x, self.w = full.x, full.w
        self.world, self.group = world, group
        self.layers = []
        for layer in full.layers:
            qkv, o, gu, dn = (layer[k] for k in ("qkv_proj", "o_proj", "gate_up_proj", "down_proj"))
            qkv_parts = (HIDDEN, (qkv.w_t.shape[1] - HIDDEN) // 2, (qkv.w_t.shape[1] - HIDDEN) // 2)
            self.layers.append({
                "qkv": tp.ColumnParallelW8A8(tp.shard_rows_of(qkv.w_t.t(), rank, world, qkv_parts),
                                             tp.shard_rows_of(qkv.scale, rank, world, qkv_parts),
                                             group=group),
                "o": tp.RowParallelW8A8(tp.shard_cols_of(o.w_t.t(), rank, world), o.scale, group=group),
                "gu": tp.ColumnParallelW8A8(tp.shard_rows_of(gu.w_t.t(), rank, world, (INTER, INTER)),
                                            tp.shard_rows_of(gu.scale, rank, world, (INTER, INTER)),
                                            group=group),
                "dn": tp.RowParallelW8A8(tp.shard_cols_of(dn.w_t.t(), rank, world), dn.scale, group=group),
            })
        del full
        torch.cuda.empty_cache()
        self.comm = comm
        self.graph: torch.cuda.CUDAGraph | None = None
        self.out: torch.Tensor | None = None

    def step(self) -> torch.Tensor:
        return self._step_peer() if self.comm is not None else self._step_nccl()

    def _step_peer(self) -> torch.Tensor:
        """The same step with the exchanges in this library's NVLink kernels: per layer
        qkv GEMM -> split-row quantiser (absmax MAX over GPUs) -> o_proj partial GEMM ->
        (int32 sum over GPUs + dequant + residual add + RMSNorm + quantiser) -> gate_up GEMM
        -> split-row SiLU-mul quantiser -> down partial GEMM -> (sum + dequant + the next
        layer's norm and quantiser).  Six kernels per layer instead of seven plus four
        collectives."""
        from int8_linear import tp

        c = self.comm
        res = self.x
        q, s, _ = add_rmsnorm_quant(self.x, None, self.w, EPS)
        q_cols = HIDDEN // self.world
        h = None
        last = len(self.layers) - 1
        for i, layer in enumerate(self.layers):
            qkv = layer["qkv"](q, s)
            q, s = tp.peer_quant_rows(c, qkv[:, :q_cols])
            acc = layer["o"].partial(q)
            q, s, res = tp.peer_allreduce_add_rmsnorm_quant(c, acc, s, layer["o"].w_s, None, res,
                                                            self.w, EPS)
            gu = layer["gu"](q, s)
            q, s = tp.peer_silu_mul_quant(c, gu)
            acc = layer["dn"].partial(q)
            if i < last:
                q, s, res = tp.peer_allreduce_add_rmsnorm_quant(c, acc, s, layer["dn"].w_s, None, res,
                                                                self.w, EPS)
            else:
                h = tp.peer_allreduce_dequant(c, acc, s, layer["dn"].w_s)
        return h

    def _step_nccl(self) -> torch.Tensor:
        from int8_linear import tp

        res = self.x
        q, s, _ = add_rmsnorm_quant(self.x, None, self.w, EPS)
        h = None
        q_cols = HIDDEN // self.world
        for i, layer in enumerate(self.layers):
            if i:
                q, s, res = add_rmsnorm_quant(h, res, self.w, EPS)
            qkv = layer["qkv"](q, s)                  # [M, 4096/g]: this rank's q | k | v
            q, s = tp.sharded_per_token_quant(qkv[:, :q_cols], group=self.group)
            h = layer["o"](q, s)                      # int32 all-reduce, dequantised once
            q, s, res = add_rmsnorm_quant(h, res, self.w, EPS)
            gu = layer["gu"](q, s)                    # [M, 12288/g]: this rank's gate | up
            q, s = tp.sharded_silu_mul_quant(gu, group=self.group)
            h = layer["dn"](q, s)
        return h

    capture = StandinDecoder.capture
