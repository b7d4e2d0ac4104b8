"""Float rounding helpers for the oracle (numpy): bf16/fp16 round trips.

Test infrastructure only (see oracle/__init__.py).
"""

from __future__ import annotations

import numpy as np


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to bfloat16 (round to nearest, ties to even), as uint16 bits."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (b & 0x7FFFFFFF) > 0x7F800000
    rounded = (b + (0x7FFF + ((b >> 16) & 1))) >> 16
    out = np.where(nan, (b >> 16) | 0x40, rounded)
    return out.astype(np.uint16)


def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 -> float32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def round_f16(x: np.ndarray) -> np.ndarray:
    """float32 -> float16 -> float32 (numpy's cast rounds to nearest even)."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values through 'bf16', 'f16' or 'f32' and back to float32."""
    if dtype == "bf16":
        return round_bf16(x)
    if dtype == "f16":
        return round_f16(x)
    if dtype == "f32":
        return np.asarray(x, dtype=np.float32)
    raise ValueError(dtype)


def to_bits(x: np.ndarray, dtype: str) -> np.ndarray:
    """float32 values rounded to dtype, as the raw storage bits (uint16 / float32)."""
    if dtype == "bf16":
        return f32_to_bf16_bits(x)
    if dtype == "f16":
        return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)
    if dtype == "f32":
        return np.asarray(x, dtype=np.float32)
    raise ValueError(dtype)
