"""Loads libint8linear_b200.so and binds its C ABI (include/int8_linear_b200.h).

There is no fallback: if the library is missing, importing the kernels raises with
the command that builds it.  Error codes become NotSupported, ValueError or
RuntimeError, exactly as the reference's launchers raise them.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libint8linear_b200.so"

OK, ENOTSUP, EINVAL, ECUDA, EWORKSPACE = 0, 1, 2, 3, 4
BF16, F16, F32, I32 = 0, 1, 2, 3


class NotSupported(Exception):
    """The kernel does not take this shape or dtype, so the caller should fall back."""


class I8LTile(ctypes.Structure):
    """Mirror of struct i8l_tile."""

    _fields_ = [(name, ctypes.c_int32) for name in (
        "swap_ab", "tok_tile", "w_tile", "stages", "ctas", "group", "split", "cluster", "store",
        "act")]


MAX_RANKS = 8
PEER_HANDLE_BYTES = 64


class I8LPeerComm(ctypes.Structure):
    """Mirror of struct i8l_peer_comm."""

    _fields_ = [("bases", ctypes.c_void_p * MAX_RANKS), ("epochs", ctypes.c_void_p),
                ("rank", ctypes.c_int32), ("world", ctypes.c_int32), ("slot_bytes", ctypes.c_int64),
                ("max_rows", ctypes.c_int32), ("timeout_ns", ctypes.c_uint64),
                ("two_shot_rows", ctypes.c_int32)]


_lib = None
_lock = threading.Lock()

_vp, _i8p, _fp = ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p
_i32, _i64, _f32, _sz = ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t

# name -> (restype, argtypes); the same list the CPU tests check against the header.
SIGNATURES = {
    "i8l_w8a8_mm": (_i32, [_i8p, _i64, _i8p, _i64, _fp, _i32, _fp, _i32, _vp, _i32, _vp, _i32, _i64,
                           _i32, _i32, _i32, ctypes.POINTER(I8LTile), _vp, _sz, _vp]),
    "i8l_w8a8_mm_quant_act": (_i32, [_vp, _i32, _i64, _i32, _i8p, _i64, _fp, _i32, _vp, _i32, _vp, _i32,
                                     _i64, _i32, _i32, _i32, ctypes.POINTER(I8LTile), _vp, _sz, _vp]),
    "i8l_rmsnorm_w8a8_mm": (_i32, [_vp, _i64, _vp, _i64, _vp, _i32, _i32, _f32, _i32, _vp, _i64, _i8p, _i64,
                                   _fp, _i32, _vp, _i32, _vp, _i32, _i64, _i32, _i32, _i32,
                                   ctypes.POINTER(I8LTile), _vp]),
    "i8l_silu_mul_w8a8_mm": (_i32, [_vp, _i64, _i32, _i32, _i32, _i8p, _i64, _fp, _i32, _vp, _i32, _vp, _i32,
                                    _i64, _i32, _i32, _i32, ctypes.POINTER(I8LTile), _vp]),
    "i8l_w8a8_mm_noalloc": (_i32, [_i8p, _i64, _i8p, _i64, _fp, _i32, _fp, _i32, _vp, _i32, _vp, _i32,
                                   _i64, _i32, _i32, _i32, ctypes.POINTER(I8LTile), _vp]),
    "i8l_workspace_size": (_sz, [_i32, _i32, _i32, ctypes.POINTER(I8LTile)]),
    "i8l_default_tile": (_i32, [_i32, _i32, _i32, ctypes.POINTER(I8LTile)]),
    "i8l_add_rmsnorm_quant": (_i32, [_vp, _i64, _vp, _i64, _vp, _i32, _i32, _i8p, _i64, _fp, _vp, _i64,
                                     _i32, _i32, _f32, _i32, _vp]),
    "i8l_silu_mul_quant": (_i32, [_vp, _i64, _i32, _i8p, _i64, _fp, _i32, _i32, _i32, _i32, _vp]),
    "i8l_quant_rows": (_i32, [_vp, _i64, _i32, _i8p, _i64, _fp, _i32, _i32, _i32, _vp]),
    "i8l_silu_mul_quant_ex": (_i32, [_vp, _i64, _i32, _i8p, _i64, _fp, _i32, _i32, _i32, _i32, _fp, _fp,
                                     _vp]),
    "i8l_quant_rows_ex": (_i32, [_vp, _i64, _i32, _i8p, _i64, _fp, _i32, _i32, _i32, _fp, _fp, _vp]),
    "i8l_dequant_i32": (_i32, [_vp, _i64, _fp, _i32, _fp, _i32, _vp, _i32, _vp, _i32, _i64, _i32, _i32,
                               _vp]),
    "i8l_last_error": (ctypes.c_char_p, []),
    "i8l_read_status": (_i32, [ctypes.POINTER(_i32)]),
    "i8l_clear_status": (_i32, []),
    "i8l_version": (ctypes.c_char_p, []),
    "i8l_set_pdl": (_i32, [_i32]),
    "i8l_get_pdl": (_i32, []),
    "i8l_peer_buffer_bytes": (_sz, [_i64, _i32]),
    "i8l_peer_alloc": (_i32, [_sz, ctypes.POINTER(_vp), _vp]),
    "i8l_peer_open": (_i32, [_vp, ctypes.POINTER(_vp)]),
    "i8l_peer_close": (_i32, [_vp]),
    "i8l_peer_free": (_i32, [_vp]),
    "i8l_tp_allreduce_dequant": (_i32, [ctypes.POINTER(I8LPeerComm), _vp, _i64, _fp, _i32, _fp, _i32,
                                        _vp, _i32, _vp, _i32, _i64, _i32, _i32, _vp]),
    "i8l_tp_allreduce_add_rmsnorm_quant": (_i32, [ctypes.POINTER(I8LPeerComm), _vp, _i64, _fp, _i32,
                                                  _fp, _i32, _vp, _i32, _vp, _i64, _vp, _i32, _i32,
                                                  _i8p, _i64, _fp, _vp, _i64, _vp, _i64, _i32, _i32,
                                                  _f32, _i32, _vp]),
    "i8l_tp_quant_rows": (_i32, [ctypes.POINTER(I8LPeerComm), _vp, _i64, _i32, _i8p, _i64, _fp, _i32,
                                 _i32, _i32, _vp]),
    "i8l_tp_silu_mul_quant": (_i32, [ctypes.POINTER(I8LPeerComm), _vp, _i64, _i32, _i8p, _i64, _fp,
                                     _i32, _i32, _i32, _i32, _vp]),
}


def load(path: Path | str | None = None) -> ctypes.CDLL:
    """The bound library (loaded once).  Raises ImportError if it was never built."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path else LIB_PATH
        if not p.exists():
            raise ImportError(
                f"{p} is missing: build the sm_100a library first with "
                "`python -m int8_linear.build` (there is no non-CUDA fallback)")
        lib = ctypes.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
            if os.environ.get("INT8_LINEAR_PDL") == "1":
                lib.i8l_set_pdl(1)
        return lib


def check(code: int) -> None:
    """Raise the exception the reference's launcher would raise for this code."""
    if code == OK:
        return
    msg = load().i8l_last_error().decode(errors="replace")
    if code == ENOTSUP:
        raise NotSupported(msg)
    if code == EINVAL:
        raise ValueError(msg)
    raise RuntimeError(f"int8_linear native call failed ({code}): {msg}")


# Called when the status word shows a kernel gave up a wait, and by clear_status():
# the GEMM module registers the re-zeroing of its split-K workspaces here.
STATUS_HOOKS: list = []


def read_status() -> int:
    """Synchronise the device and return the kernels' status word (0 = clean).  A
    non-zero word also re-zeroes the cached split-K workspaces (STATUS_HOOKS): a kernel
    that gave up a wait may have left partial sums in them."""
    v = _i32(0)
    check(load().i8l_read_status(ctypes.byref(v)))
    if v.value:
        for hook in STATUS_HOOKS:
            hook()
    return int(v.value)


def clear_status() -> None:
    """Reset the status word and re-zero the cached split-K workspaces."""
    check(load().i8l_clear_status())
    for hook in STATUS_HOOKS:
        hook()


def set_pdl(enable: bool) -> None:
    """Launch every kernel with programmatic dependent launch (see i8l_set_pdl): a kernel
    may start while the previous one in the stream runs, and GEMMs prefetch weight tiles
    before waiting for it.  Only for weights that the preceding kernel never writes."""
    check(load().i8l_set_pdl(1 if enable else 0))


def pdl_enabled() -> bool:
    return bool(load().i8l_get_pdl())
