"""Helpers for the GPU parity tests: seeded CPU inputs, copies to the device, and
numpy views of device results for the oracle comparison."""

from __future__ import annotations

import numpy as np
import torch


def ints(shape, seed, low=-127, high=128) -> torch.Tensor:
    """Seeded int8 values on the GPU (drawn on the CPU so the oracle sees the same)."""
    g = torch.Generator().manual_seed(seed)
    return torch.randint(low, high, shape, dtype=torch.int8, generator=g).cuda()


def rand(shape, seed, scale=1.0, dtype=torch.bfloat16) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(dtype).cuda()


def offset_ints(shape, seed) -> torch.Tensor:
    """int8 values stored one byte into their buffer, so the data pointer is odd."""
    flat = ints((shape[0] * shape[1] + 1,), seed)
    return flat[1:].view(shape)


def np_(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.float().numpy()
    return t.numpy()


def bits(t: torch.Tensor) -> np.ndarray:
    """Raw storage bits of a 16-bit float tensor (uint16), or the values otherwise."""
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()
