"""W8A8 int8 matmul with the dequantisation fused in, on B200 (sm_100a).

    C[M, N] = (A_q[M, K] @ W_q[K, N]) * scale_a[M] * scale_b[N] + bias[N]

Same Python API as the reference module int8_linear/kernel.py (AshrithaG/int8-linear):
w8a8_mm, Config, NotSupported, default_config, tuned_config, choose_config.  The
work is done by the hand-written sm_100a kernel in csrc/gemm_sm100.cu (tcgen05
kind::i8 MMA, TMEM accumulators, TMA pipeline, fused epilogue), reached through the
C ABI of libint8linear_b200.so; there is no Triton and no CPU path.

W_q is the transposed [K, N] view of an [N, K] nn.Linear weight (strides (1, K)),
which is how vLLM passes it; both operands are then K-contiguous, the layout the
tensor cores read.  The launch goes straight from Python to the C ABI on torch's
current stream, so there is no JIT dispatch to cache: `cached_launch` is accepted
for compatibility and has no effect.  Under torch.compile, call the kernel through
the custom op in int8_linear/vllm_patch.py rather than tracing into it.
"""

from __future__ import annotations

import ctypes
import json
from dataclasses import dataclass, replace
from functools import lru_cache
from pathlib import Path

import torch

from int8_linear import _native
from int8_linear._native import NotSupported

TUNED_PATH = Path(__file__).with_name("tuned_configs.json")
TOKEN_TILES = (16, 32, 64, 128, 256)
GEMV_TOKENS = (1, 2, 4, 8, 16)   # token counts of the CUDA-core tiles (split 5)
# Split-K workspace kept per (device, stream); kernels leave it zero-filled.  The
# largest plan needs (SMs - 1) slots of 128 x 256 int32 plus counters, ~19 MB on
# 148 SMs, so one allocation covers every call.
WORKSPACE_BYTES = 32 << 20

__all__ = ["Config", "NotSupported", "default_config", "tuned_config", "choose_config", "w8a8_mm",
           "w8a8_mm_quant_act", "rmsnorm_w8a8_mm", "silu_mul_w8a8_mm"]


@dataclass(frozen=True)
class Config:
    """One B200 GEMM tiling.

    bm      token tile.  With swap_ab the tokens are the MMA N side, bm in
            {16, 32, 64, 128, 256}; without, they fill the 128-row MMA M side, bm = 128.
    bn      weight tile: 128 with swap_ab (the MMA M side), else 128 or 256.
    bk      K bytes per pipeline stage; 128 (one 128-byte swizzle row).
    warps   warps per CTA: one TMA producer, one MMA issuer, four epilogue warps.
    stages  shared-memory ring depth, 0 for the most that fits.
    group_m 128-row tiles walked together so concurrent CTAs share tiles in L2.
    swap_ab None picks swap_ab for bm != 128.
    split   how K is shared out; int32 partial sums are always reduced exactly, so every
            choice gives the same bits: 0 the library's choice, 1 whole tiles, 2
            stream-K over the SMs (reduced in a workspace), 3 cluster split-K (the CTAs
            of a thread-block cluster split a tile's K and reduce over distributed
            shared memory; swap_ab tiles, each CTA finishing one in `cluster` of the
            tile's 16-column chunks from the others' partial sums; without swap_ab,
            narrow 128 x 256 tiles for batches of <= 16 tokens, and 128-token tiles of
            128 or 256 weight rows for larger batches, the weight on the MMA's N side in
            both), 4 CTA pairs (two SMs
            per 256 x 256 tile with 256-row tcgen05 MMAs; 128 x 256 tiles, no swap_ab),
            5 CUDA-core tiles for decode batches of at most 16 tokens: bm in
            (1, 2, 4, 8, 16) is the most tokens, bn = 0; each CTA owns whole output columns (int8 dot
            products with dp4a, no split-K), its weight rows streamed into shared memory
            by 1-D bulk copies that start before the dependency wait.
    ctas    persistent CTAs, 0 for one per SM.
    cluster CTAs per cluster for split=3, 0 for the library's choice.
    store   output path: 0 the library's choice, 1 TMA stores, 2 plain stores.
    act     activation path of swap_ab tiles: 0 the library's choice, 1 TMA loads, 2
            plain loads right after the dependency wait (M <= bm, one tile or cluster
            segment per CTA, and all of that segment's k-blocks in the ring at once).
    """

    bm: int
    bn: int
    bk: int = 128
    warps: int = 6
    stages: int = 0
    group_m: int = 8
    swap_ab: bool | None = None
    split: int = 0
    ctas: int = 0
    cluster: int = 0
    store: int = 0
    act: int = 0

    @property
    def swapped(self) -> bool:
        if self.split == 5:
            return False
        return self.bm != 128 if self.swap_ab is None else bool(self.swap_ab)

    @property
    def name(self) -> str:
        if self.split == 5:
            return f"gemv m{self.bm} s{self.stages}" + (f" c{self.ctas}" if self.ctas else "")
        tail = (" swap" if self.swapped else "") + {0: "", 1: " whole", 2: " sk", 3: " cl", 4: " pair"}.get(
            self.split, f" split{self.split}")
        tail += str(self.cluster) if self.split == 3 and self.cluster else ""
        tail += f" c{self.ctas}" if self.ctas else ""
        tail += {1: " tma", 2: " direct"}.get(self.store, "")
        tail += {1: " act-tma", 2: " act-ld"}.get(self.act, "")
        return f"{self.bm}x{self.bn}x{self.bk} w{self.warps} s{self.stages} g{self.group_m}{tail}"

    def check(self) -> None:
        """Raise NotSupported unless a B200 kernel exists for this tiling."""
        if self.split == 5:
            if self.bm not in GEMV_TOKENS or self.bn != 0 or self.stages < 0 or self.ctas < 0:
                raise NotSupported(f"{self.name}: CUDA-core tiles take bm in {GEMV_TOKENS}, bn 0")
            return
        if self.bk != 128 or self.warps != 6:
            raise NotSupported(f"{self.name}: B200 tiles use bk=128 and 6 warps")
        if self.swapped:
            if self.bm not in TOKEN_TILES or self.bn != 128:
                raise NotSupported(f"{self.name}: swap_ab tiles are bm in {TOKEN_TILES} x bn 128")
        elif self.bm != 128 or self.bn not in (128, 256):
            raise NotSupported(f"{self.name}: tiles are bm 128 x bn in (128, 256)")
        if self.stages < 0 or self.stages == 1 or self.group_m < 1 or self.split not in (0, 1, 2, 3, 4, 5):
            raise NotSupported(f"{self.name}: bad stages/group_m/split")
        if self.store not in (0, 1, 2) or self.act not in (0, 1, 2):
            raise NotSupported(f"{self.name}: store and act must be 0, 1 or 2")
        if self.act == 2 and not self.swapped:
            raise NotSupported(f"{self.name}: direct activation loads take swap_ab tiles")
        if self.split == 3 and not 0 <= self.cluster <= 8:
            raise NotSupported(f"{self.name}: clusters hold at most 8 CTAs")

        if self.split == 4 and (self.swapped or self.bn != 256):
            raise NotSupported(f"{self.name}: CTA pairs take 128 x 256 tiles without swap_ab")

    def as_tile(self) -> _native.I8LTile:
        if self.split == 5:
            return _native.I8LTile(swap_ab=0, tok_tile=self.bm, w_tile=0, stages=self.stages,
                                   ctas=self.ctas, group=1, split=5)
        return _native.I8LTile(
            swap_ab=1 if self.swapped else 0, tok_tile=self.bm if self.swapped else 128,
            w_tile=128 if self.swapped else self.bn, stages=self.stages, ctas=self.ctas,
            group=self.group_m, split=self.split, cluster=self.cluster, store=self.store,
            act=self.act)


def default_config(m: int, n: int, k: int) -> Config:
    """The untuned choice.  Batches of at most 4 tokens, and of at most 8 on weights up to
    16 MB, take the CUDA-core tiles (split 5; measured faster than every tensor-core tiling
    there on B200).  Other decode batches (M <= 256) put the weight on the 128-row
    MMA side and the tokens on the narrow side, the smallest token tile that holds
    M; larger batches use 128 x 256 tiles.  The library then splits K inside
    thread-block clusters when decode tiles would leave SMs idle (never by stream-K,
    which measured slower on every shape tried).  Prefill with K >= 4096 uses CTA pairs
    (split 4).  Batches of
    one or two tokens on moderate weights (K 1024..6144, N <= 8192) take narrow tiles
    instead: 256 weight rows per MMA, K split over a cluster of up to 8 CTAs with at
    least two 128-wide k-blocks each (measured faster there on B200; larger weights
    have too few 256-row tiles to fill the SMs)."""
    if m <= 4 or (m <= 8 and n * k <= 16 << 20):
        return Config(next(t for t in GEMV_TOKENS if t >= m), 0, split=5)
    if m <= 256:
        return Config(next(t for t in TOKEN_TILES if t >= m), 128)
    # Prefill: the wider tile unless the narrower one fills the SMs clearly better.
    sms = 148
    def waves_eff(bn):
        tiles = -(-m // 128) * -(-n // bn)
        waves = -(-tiles // sms)
        return tiles / (waves * sms)
    if waves_eff(256) < 0.8 * waves_eff(128):
        return Config(128, 128)
    # Long K: pairs of SMs per 256 x 256 tile (cta_group::2) halve each SM's weight fill.
    return Config(128, 256, split=4) if k >= 4096 else Config(128, 256)


@lru_cache(maxsize=None)
def _tuned_table(device_name: str) -> dict:
    tables = json.loads(TUNED_PATH.read_text()) if TUNED_PATH.exists() else {}
    return tables.get(device_name, {})


def tuned_config(m: int, n: int, k: int) -> Config | None:
    """The fastest measured config for this GPU and shape, from the largest tuned
    batch bucket at or below M, or None if nothing has been tuned."""
    table = _tuned_table(torch.cuda.get_device_name()).get(f"{k}x{n}", {})
    fits = [int(bucket) for bucket in table if int(bucket) <= m]
    return Config(**table[str(max(fits))]["config"]) if fits else None


_chosen: dict[tuple[int, int, int, int], Config] = {}


def _fits(cfg: Config, m: int, n: int, k: int) -> Config:
    """cfg adapted to M when a table bucket's tiling cannot hold it: a CUDA-core tile for
    fewer tokens than M takes the next larger token count (up to 16), else the default."""
    if cfg.split == 5 and m > cfg.bm:
        bigger = [t for t in GEMV_TOKENS if t >= m]
        return replace(cfg, bm=bigger[0]) if bigger else default_config(m, n, k)
    return cfg


def choose_config(m: int, n: int, k: int) -> Config:
    """tuned_config, else default_config, remembered per device and shape."""
    key = (torch.cuda.current_device(), m, n, k)
    cfg = _chosen.get(key)
    if cfg is None:
        cfg = _chosen[key] = _fits(tuned_config(m, n, k) or default_config(m, n, k), m, n, k)
    return cfg


_DTYPE_CODE = {torch.bfloat16: _native.BF16, torch.float16: _native.F16, torch.float32: _native.F32}
_workspaces: dict[tuple[int, int], torch.Tensor] = {}
_capture_workspaces: dict[int, torch.Tensor] = {}
_tiles: dict[Config, _native.I8LTile] = {}
# The current stream's raw handle without building a torch.cuda.Stream object (the host
# cost of an eager call is a few microseconds, so each one counts).
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def current_stream(device_index: int) -> int:
    if _raw_stream is not None:
        return _raw_stream(device_index)
    return torch.cuda.current_stream(device_index).cuda_stream


def _tile_of(cfg: Config) -> _native.I8LTile:
    """The C tile struct of a validated config (checked and built once per config)."""
    tile = _tiles.get(cfg)
    if tile is None:
        cfg.check()
        tile = _tiles[cfg] = cfg.as_tile()
    return tile


def _zeroed(index: int) -> torch.Tensor:
    return torch.zeros(WORKSPACE_BYTES, dtype=torch.uint8, device=torch.device("cuda", index))


def workspace(device: torch.device | int, stream: int) -> torch.Tensor:
    """The zero-filled split-K workspace for calls on this device and stream.

    Eager calls get one workspace per (device, stream), allocated on the first call.
    Calls captured into a CUDA graph share one workspace per device, allocated and
    zeroed (together with the first eager one) outside any capture: a buffer created
    inside a capture would come from that graph's private pool, and its zero fill would
    be a node of that one graph, done only when that graph is replayed.  So the first
    GEMM on a device must not be inside a capture (a warm-up call first, as graph capture
    needs anyway), and graphs captured on one device must not be replayed concurrently
    on different streams.  Kernels leave a workspace zeroed; reset_workspaces() zeroes
    them all again after a kernel gave up a wait (i8l_read_status)."""
    index = device if isinstance(device, int) else device.index
    key = (index, stream)
    ws = _workspaces.get(key)
    if ws is not None:
        return ws
    if torch.cuda.is_current_stream_capturing():
        ws = _capture_workspaces.get(index)
        if ws is None:
            raise RuntimeError(
                f"the first int8_linear GEMM on cuda:{index} is being captured into a CUDA graph: "
                "make one call outside the capture first (a warm-up), so the split-K workspace "
                "is allocated and zeroed before it")
    else:
        if index not in _capture_workspaces:
            _capture_workspaces[index] = _zeroed(index)
        ws = _zeroed(index)
    _workspaces[key] = ws
    return ws


def reset_workspaces() -> None:
    """Zero every cached split-K workspace again (and wait for it).  Kernels leave their
    slots and counters zeroed when they finish; one whose bounded wait gave up may not
    have, and later split-K calls would then add into stale sums."""
    for ws in {id(w): w for w in (*_workspaces.values(), *_capture_workspaces.values())}.values():
        with torch.cuda.device(ws.device):
            ws.zero_()
            torch.cuda.synchronize()


_native.STATUS_HOOKS.append(reset_workspaces)


def _aligned_rows(t: torch.Tensor) -> torch.Tensor:
    """t itself when its rows start on 16-byte boundaries (what TMA needs), else an
    aligned contiguous copy.  The reference takes any pointer; this keeps odd
    pointers exact at the cost of one copy."""
    if t.stride(1) == 1 and t.data_ptr() % 16 == 0 and t.stride(0) % 16 == 0:
        return t
    out = torch.empty(t.shape, dtype=t.dtype, device=t.device)
    out.copy_(t)
    return out


def w8a8_mm(
    a_q: torch.Tensor,
    b_q: torch.Tensor,
    scale_a: torch.Tensor,
    scale_b: torch.Tensor,
    out_dtype: torch.dtype = torch.bfloat16,
    bias: torch.Tensor | None = None,
    *,
    config: Config | None = None,
    raw: bool = False,
    cached_launch: bool = True,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """(A_q @ B_q) * scale_a * scale_b + bias, for int8 A_q [M, K] and B_q [K, N].

    scale_a is per row ([M] or [M, 1]) or a scalar, scale_b per column ([N] or
    [N, 1]) or a scalar, both float32.  With raw=True the exact int32 product is
    returned and the scales and bias are ignored.  Raises NotSupported for what the
    kernel does not take (the caller may fall back) and ValueError for inconsistent
    arguments, as the reference does (int8_linear/kernel.py:221-240).  `out` (an
    addition to the reference's signature) is an [M, N] tensor of the output dtype
    with contiguous rows to write into instead of a new one.
    """
    del cached_launch  # launches never go through a JIT dispatch here
    if a_q.dtype != torch.int8 or b_q.dtype != torch.int8:
        raise NotSupported(f"int8 operands only, got {a_q.dtype} and {b_q.dtype}")
    if a_q.dim() != 2 or b_q.dim() != 2 or a_q.shape[1] != b_q.shape[0]:
        raise ValueError(f"cannot multiply {tuple(a_q.shape)} by {tuple(b_q.shape)}")
    m, k = a_q.shape
    n = b_q.shape[1]
    tile = _tile_of(config or choose_config(m, n, k))
    if k % 16:
        raise NotSupported(f"K={k} must be a multiple of 16 (TMA rows of 16-byte granules)")
    if n > 1 and b_q.stride(0) != 1:
        raise NotSupported("B_q must be the K-contiguous [K, N] view of an [N, K] weight")
    sa = scale_a if scale_a.is_contiguous() else scale_a.contiguous()
    sb = scale_b if scale_b.is_contiguous() else scale_b.contiguous()
    if sa.dtype != torch.float32 or sb.dtype != torch.float32:
        raise NotSupported(f"float32 scales only, got {sa.dtype} and {sb.dtype}")
    if sa.numel() not in (1, m) or sb.numel() not in (1, n):
        raise ValueError(f"scale sizes {sa.numel()} and {sb.numel()} fit neither {m} nor {n}")
    if bias is not None and tuple(bias.shape) != (n,):
        raise ValueError(f"bias must have shape ({n},), got {tuple(bias.shape)}")
    if bias is not None:
        if bias.dtype not in _DTYPE_CODE:
            raise NotSupported(f"bias dtype {bias.dtype} not supported")
        bias = bias.contiguous()
    if not raw and out_dtype not in _DTYPE_CODE:
        raise NotSupported(f"output dtype {out_dtype} not supported")
    if not (a_q.is_cuda and b_q.is_cuda and sa.is_cuda and sb.is_cuda):
        raise ValueError("w8a8_mm runs on a CUDA device; got tensors on "
                         f"{a_q.device}, {b_q.device}, {sa.device}, {sb.device}")

    want_dtype = torch.int32 if raw else out_dtype
    if out is None:
        out = torch.empty((m, n), dtype=want_dtype, device=a_q.device)
    elif tuple(out.shape) != (m, n) or out.dtype != want_dtype or out.device != a_q.device \
            or (n > 1 and out.stride(1) != 1):
        raise ValueError(f"out must be a {want_dtype} [{m}, {n}] tensor with contiguous rows on "
                         f"{a_q.device}, got {out.dtype} {tuple(out.shape)} strides {out.stride()}")
    if m == 0 or n == 0:
        return out
    a = _aligned_rows(a_q)
    # The weight's [N, K] rows are b_q's columns: row stride b_q.stride(1).
    wp, ldw = b_q.data_ptr(), b_q.stride(1)
    if b_q.stride(0) != 1 or wp % 16 or ldw % 16:
        w = _aligned_rows(b_q.t())
        wp, ldw = w.data_ptr(), w.stride(0)
    lib = _native.load()
    dev = a_q.get_device()
    stream = current_stream(dev)
    ws = workspace(dev, stream)
    if dev != torch.cuda.current_device():
        with torch.cuda.device(dev):
            code = _launch(lib, a, wp, ldw, sa, sb, bias, out, raw, out_dtype, m, n, k, tile, ws, stream)
    else:
        code = _launch(lib, a, wp, ldw, sa, sb, bias, out, raw, out_dtype, m, n, k, tile, ws, stream)
    _native.check(code)
    return out


def _launch(lib, a, wp, ldw, sa, sb, bias, out, raw, out_dtype, m, n, k, tile, ws, stream) -> int:
    return lib.i8l_w8a8_mm(
        a.data_ptr(), a.stride(0), wp, ldw,
        sa.data_ptr(), int(sa.numel() > 1), sb.data_ptr(), int(sb.numel() > 1),
        bias.data_ptr() if bias is not None else None,
        _DTYPE_CODE[bias.dtype] if bias is not None else 0,
        out.data_ptr(), _native.I32 if raw else _DTYPE_CODE[out_dtype], out.stride(0),
        m, n, k, ctypes.byref(tile), ws.data_ptr(), ws.numel(), stream)


def fused_act_config(cfg: Config) -> Config | None:
    """The tiling of cfg that w8a8_mm_quant_act can fuse into: a CUDA-core tile itself, the
    same swap_ab tiling with direct activation loads, or None for other tiles."""
    if cfg.split == 5:
        return cfg
    if not cfg.swapped:
        return None
    return cfg if cfg.act == 2 else replace(cfg, act=2)


def _fused_candidates(m: int, n: int, k: int) -> list[Config]:
    """Tilings w8a8_mm_quant_act tries, in order, when the caller names none: the table's
    CUDA-core tile (its prologue quantises), or the table's tile with direct loads, then
    cluster split-K tilings of the smallest token tile that holds M, then whole tiles,
    one per CTA."""
    out = []
    chosen = choose_config(m, n, k)
    if chosen.split == 5:
        return [chosen]
    base = fused_act_config(chosen)
    if base is not None:
        out.append(base)
    if m <= 64:
        tn = next(t for t in TOKEN_TILES if t >= m)
        out += [Config(tn, 128, split=3, cluster=c, act=2) for c in (4, 8, 3, 2, 6)]
        out.append(Config(tn, 128, split=1, act=2, ctas=-(-n // 128)))
    return out


_fused_chosen: dict[tuple[int, int, int, int], Config | None] = {}


def w8a8_mm_quant_act(
    x: torch.Tensor,
    b_q: torch.Tensor,
    scale_b: torch.Tensor,
    out_dtype: torch.dtype = torch.bfloat16,
    bias: torch.Tensor | None = None,
    *,
    config: Config | None = None,
    precise_div: bool = True,
    raw: bool = False,
) -> torch.Tensor:
    """w8a8_mm of x's dynamic per-token int8 quantisation: the same bits as
    `q, s = fused_quant.per_token_quant(x, precise_div); w8a8_mm(q, b_q, s, scale_b, ...)`.

    x is a bf16/fp16 [M, K] activation with contiguous, 16-byte aligned rows (a column
    slice of a wider matrix is fine).  Where a tiling with direct activation loads takes
    the problem (decode batches on swap_ab tiles), one kernel quantises x while loading
    it; otherwise the two steps above run.  With config=None the first of the table's
    tiling and a few cluster split-K tilings that the library accepts is used (and
    remembered per shape).  This is the reference's o_proj input path
    (bench/fuse_quant.py:234: vLLM's scaled_int8_quant, then w8a8_mm) in one launch.
    """
    if x.dtype not in (torch.bfloat16, torch.float16) or x.dim() != 2 or x.stride(1) != 1:
        raise NotSupported("x must be a 2-D bf16/fp16 activation with contiguous rows")
    if b_q.dtype != torch.int8 or b_q.dim() != 2 or x.shape[1] != b_q.shape[0]:
        raise ValueError(f"cannot multiply {tuple(x.shape)} by {tuple(b_q.shape)}")
    m, k = x.shape
    n = b_q.shape[1]
    fusable = (m > 0 and n > 0 and k % 16 == 0 and x.is_cuda and x.data_ptr() % 16 == 0
               and (x.stride(0) * 2) % 16 == 0 and b_q.stride(0) == 1 and b_q.data_ptr() % 16 == 0
               and b_q.stride(1) % 16 == 0)
    if fusable:
        sb = scale_b if scale_b.is_contiguous() else scale_b.contiguous()
        if sb.dtype != torch.float32 or sb.numel() not in (1, n):
            raise ValueError(f"scale_b must hold 1 or {n} float32 values")
        if bias is not None:
            if tuple(bias.shape) != (n,):
                raise ValueError(f"bias must have shape ({n},), got {tuple(bias.shape)}")
            if bias.dtype not in _DTYPE_CODE:
                raise NotSupported(f"bias dtype {bias.dtype} not supported")
            bias = bias.contiguous()
        if not raw and out_dtype not in _DTYPE_CODE:
            raise NotSupported(f"output dtype {out_dtype} not supported")
        dev = x.get_device()
        key = (dev, m, n, k)
        if config is not None:
            tries = [c for c in (fused_act_config(config),) if c is not None]
        elif key in _fused_chosen:
            tries = [c for c in (_fused_chosen[key],) if c is not None]
        else:
            tries = _fused_candidates(m, n, k)
        out = torch.empty((m, n), dtype=torch.int32 if raw else out_dtype, device=x.device)
        lib = _native.load()
        stream = current_stream(dev)
        ws = workspace(dev, stream)
        for cfg in tries:
            code = lib.i8l_w8a8_mm_quant_act(
                x.data_ptr(), _native.BF16 if x.dtype == torch.bfloat16 else _native.F16,
                x.stride(0), int(bool(precise_div)), b_q.data_ptr(), b_q.stride(1), sb.data_ptr(),
                int(sb.numel() > 1), bias.data_ptr() if bias is not None else None,
                _DTYPE_CODE[bias.dtype] if bias is not None else 0,
                out.data_ptr(), _native.I32 if raw else _DTYPE_CODE[out_dtype], out.stride(0),
                m, n, k, ctypes.byref(_tile_of(cfg)), ws.data_ptr(), ws.numel(), stream)
            if code != _native.ENOTSUP:
                _native.check(code)
                if config is None:
                    _fused_chosen[key] = cfg
                return out
        if config is None:
            _fused_chosen[key] = None
    from int8_linear.fused_quant import per_token_quant

    q, s = per_token_quant(x, precise_div)
    return w8a8_mm(q, b_q, s, scale_b, out_dtype, bias, config=config, raw=raw)


def dequant_i32(acc: torch.Tensor, scale_a: torch.Tensor, scale_b: torch.Tensor,
                out_dtype: torch.dtype = torch.bfloat16, bias: torch.Tensor | None = None) -> torch.Tensor:
    """cast(((float(acc) * scale_a) * scale_b) + bias) for an int32 [M, N] product made
    elsewhere (e.g. summed over the GPUs of a row-parallel layer): the GEMM epilogue's
    arithmetic, so the result equals w8a8_mm on the whole product bit for bit."""
    if acc.dtype != torch.int32 or acc.dim() != 2 or acc.stride(1) != 1:
        raise ValueError("acc must be a 2-D int32 tensor with contiguous rows")
    m, n = acc.shape
    sa, sb = scale_a.reshape(-1).contiguous(), scale_b.reshape(-1).contiguous()
    if sa.numel() not in (1, m) or sb.numel() not in (1, n):
        raise ValueError(f"scale sizes {sa.numel()} and {sb.numel()} fit neither {m} nor {n}")
    if out_dtype not in _DTYPE_CODE or (bias is not None and bias.dtype not in _DTYPE_CODE):
        raise NotSupported("bf16/fp16/fp32 output and bias only")
    bias = bias.contiguous() if bias is not None else None
    out = torch.empty((m, n), dtype=out_dtype, device=acc.device)
    if m and n:
        _native.check(_native.load().i8l_dequant_i32(
            acc.data_ptr(), acc.stride(0), sa.data_ptr(), int(sa.numel() > 1), sb.data_ptr(),
            int(sb.numel() > 1), bias.data_ptr() if bias is not None else None,
            _DTYPE_CODE[bias.dtype] if bias is not None else 0, out.data_ptr(), _DTYPE_CODE[out_dtype],
            out.stride(0), m, n, torch.cuda.current_stream(acc.device).cuda_stream))
    return out


def _gemv_fused_config(m: int, n: int, k: int, config: Config | None) -> Config | None:
    """The CUDA-core tile a fused-quantiser call runs on, or None to run the two steps:
    the caller's tiling if it is one, else the library's choice for the shape if it is one."""
    cfg = config if config is not None else choose_config(m, n, k)
    return cfg if cfg.split == 5 else None


def _gemv_args(b_q, scale_b, bias, out_dtype, n):
    if b_q.dtype != torch.int8 or b_q.dim() != 2:
        raise NotSupported("b_q must be a 2-D int8 weight")
    sb = scale_b if scale_b.is_contiguous() else scale_b.contiguous()
    if sb.dtype != torch.float32 or sb.numel() not in (1, n):
        raise ValueError(f"scale_b must hold 1 or {n} float32 values")
    if bias is not None:
        if tuple(bias.shape) != (n,):
            raise ValueError(f"bias must have shape ({n},), got {tuple(bias.shape)}")
        if bias.dtype not in _DTYPE_CODE:
            raise NotSupported(f"bias dtype {bias.dtype} not supported")
        bias = bias.contiguous()
    if out_dtype not in _DTYPE_CODE:
        raise NotSupported(f"output dtype {out_dtype} not supported")
    return sb, bias


def rmsnorm_w8a8_mm(x: torch.Tensor, residual: torch.Tensor | None, weight: torch.Tensor, eps: float,
                    b_q: torch.Tensor, scale_b: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16,
                    bias: torch.Tensor | None = None, *, precise_div: bool = True,
                    config: Config | None = None):
    """`q, s, rout = add_rmsnorm_quant(x, residual, weight, eps, precise_div)` followed by
    `w8a8_mm(q, b_q, s, scale_b, out_dtype, bias)`: returns (out, rout), the same bits.

    For decode batches on a CUDA-core tile (the library's choice for M <= 8 on most
    shapes, or `config`), one kernel does both: every CTA normalises and quantises the
    batch in its prologue (the standalone kernel's thread layout and reduction order)
    and the int8 activation never reaches HBM.  Otherwise the two steps run.  This is the
    reference's decoder-layer pair, add_rmsnorm_quant then the int8 linear
    (int8_linear/vllm_fuse_patch.py:41-52)."""
    from int8_linear.fused_quant import _WEIGHT, add_rmsnorm_quant

    m, k = x.shape
    n = b_q.shape[1]
    cfg = _gemv_fused_config(m, n, k, config) if x.dim() == 2 and b_q.shape[0] == k else None
    if cfg is not None and m > 0 and n > 0 and x.dtype in (torch.bfloat16, torch.float16) \
            and x.is_cuda and x.stride(1) == 1 and weight.dtype in _WEIGHT and weight.numel() == k \
            and b_q.stride(0) == 1:
        sb, bias = _gemv_args(b_q, scale_b, bias, out_dtype, n)
        w = weight.contiguous()
        rout = None
        if residual is not None:
            if residual.shape != x.shape or residual.dtype != x.dtype:
                raise ValueError("residual must match x in shape and dtype")
            rout = torch.empty_like(x)
        out = torch.empty((m, n), dtype=out_dtype, device=x.device)
        dev = x.get_device()
        code = _native.load().i8l_rmsnorm_w8a8_mm(
            x.data_ptr(), x.stride(0),
            residual.data_ptr() if residual is not None else None,
            residual.stride(0) if residual is not None else 0,
            w.data_ptr(), _native.BF16 if x.dtype == torch.bfloat16 else _native.F16, _WEIGHT[w.dtype],
            float(eps), int(bool(precise_div)), rout.data_ptr() if rout is not None else None,
            rout.stride(0) if rout is not None else 0, b_q.data_ptr(), b_q.stride(1), sb.data_ptr(),
            int(sb.numel() > 1), bias.data_ptr() if bias is not None else None,
            _DTYPE_CODE[bias.dtype] if bias is not None else 0, out.data_ptr(), _DTYPE_CODE[out_dtype],
            out.stride(0), m, n, k, ctypes.byref(_tile_of(cfg)), current_stream(dev))
        if code != _native.ENOTSUP:
            _native.check(code)
            return out, rout
    q, s, rout = add_rmsnorm_quant(x.contiguous(), residual, weight, eps, precise_div)
    return w8a8_mm(q, b_q, s, scale_b, out_dtype, bias, config=config), rout


def silu_mul_w8a8_mm(gate_up: torch.Tensor, b_q: torch.Tensor, scale_b: torch.Tensor,
                     out_dtype: torch.dtype = torch.bfloat16, bias: torch.Tensor | None = None, *,
                     precise_div: bool = True, round_silu: bool = False,
                     config: Config | None = None) -> torch.Tensor:
    """`q, s = silu_mul_quant(gate_up, precise_div, round_silu)` followed by
    `w8a8_mm(q, b_q, s, scale_b, out_dtype, bias)`, the same bits; one kernel on a
    CUDA-core tile (SiLU-and-mul and the quantiser in every CTA's prologue), else the two
    steps.  The reference's MLP pair, silu_mul_quant then down_proj
    (int8_linear/vllm_fuse_patch.py:55-59)."""
    from int8_linear.fused_quant import silu_mul_quant

    m, i2 = gate_up.shape
    k = i2 // 2
    n = b_q.shape[1]
    cfg = _gemv_fused_config(m, n, k, config) if b_q.shape[0] == k else None
    if cfg is not None and m > 0 and n > 0 and gate_up.dtype in (torch.bfloat16, torch.float16) \
            and gate_up.is_cuda and gate_up.stride(1) == 1 and b_q.stride(0) == 1:
        sb, bias = _gemv_args(b_q, scale_b, bias, out_dtype, n)
        out = torch.empty((m, n), dtype=out_dtype, device=gate_up.device)
        dev = gate_up.get_device()
        code = _native.load().i8l_silu_mul_w8a8_mm(
            gate_up.data_ptr(), gate_up.stride(0),
            _native.BF16 if gate_up.dtype == torch.bfloat16 else _native.F16, int(bool(precise_div)),
            int(bool(round_silu)), b_q.data_ptr(), b_q.stride(1), sb.data_ptr(), int(sb.numel() > 1),
            bias.data_ptr() if bias is not None else None, _DTYPE_CODE[bias.dtype] if bias is not None else 0,
            out.data_ptr(), _DTYPE_CODE[out_dtype], out.stride(0), m, n, k,
            ctypes.byref(_tile_of(cfg)), current_stream(dev))
        if code != _native.ENOTSUP:
            _native.check(code)
            return out
    q, s = silu_mul_quant(gate_up.contiguous(), precise_div, round_silu)
    return w8a8_mm(q, b_q, s, scale_b, out_dtype, bias, config=config)
