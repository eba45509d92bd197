"""bfloat16 helpers for the oracle (test infrastructure only).

bf16 values are carried as their uint16 bit patterns, so that the oracle never
depends on a framework's bf16 rounding: every rounding step is written out
here (round to nearest, ties to even, as the CUDA `__float2bfloat16_rn` and
MLX's `astype(bfloat16)` do).
"""

from __future__ import annotations

import numpy as np


def f32_to_bf16_bits(x) -> np.ndarray:
    """float32 array -> uint16 bf16 bit patterns, round to nearest even.

    NaNs are kept quiet NaNs; infinities stay infinities."""
    f = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = f.view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    r = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(f)
    if nan.any():
        r = r.copy()
        r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(b) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32 (exact)."""
    b = np.ascontiguousarray(np.asarray(b, dtype=np.uint16))
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_bf16(x) -> np.ndarray:
    """float64/float32 -> nearest bf16 value, returned as float32.

    float64 input is first rounded to float32 (as a float32 kernel would hold
    it), then to bf16."""
    return bf16_bits_to_f32(f32_to_bf16_bits(np.asarray(x, dtype=np.float32)))


def to_torch_bf16(bits):
    """uint16 bf16 bits (numpy) -> torch.bfloat16 tensor on the CPU (no rounding)."""
    import torch

    a = np.ascontiguousarray(np.asarray(bits, dtype=np.uint16))
    return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16)


def from_torch_bf16(t) -> np.ndarray:
    """torch.bfloat16 tensor -> uint16 bf16 bits (numpy)."""
    import torch

    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
