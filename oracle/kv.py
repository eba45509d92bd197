"""8-bit KV-cache formats, restated on the CPU. TEST INFRASTRUCTURE ONLY.

Two formats:
  * REF_Q8_ROW — the reference's own Q8KVCache (mlx-tree-spec
    src/mlx_tree_spec/kv8.py:39-43, 95-148): each (token, head) row of D values
    is int8 = clip(rint(x / s), -127, 127) with one float32 scale
    s = max(max|x| / 127, 1e-6). Value = int8 * s.
  * MLX_Q8_G64 — mlx-lm's quantized cache, `mx.quantize(bits=8,
    group_size=64)` per K/V row: uint32 words of four 8-bit codes (lowest byte
    first, by analogy with the 4-bit format; not pinned by the reference),
    bf16 scale and bias per 64 values. Value = s * q + b.
"""

from __future__ import annotations

import numpy as np

from .bf16 import bf16_bits_to_f32
from .qmm import pack_bits, quantize, unpack_bits


def quantize_rows(x: np.ndarray):
    """float [..., D] -> (int8 [..., D], float32 scales [...]) as kv8.quantize_rows."""
    xf = np.asarray(x, dtype=np.float32)
    s = np.maximum(np.abs(xf).max(axis=-1, keepdims=True) / np.float32(127.0), np.float32(1e-6)).astype(np.float32)
    q = np.clip(np.rint(xf / s), -127, 127).astype(np.int8)
    return q, s[..., 0]


def dequant_rows(q: np.ndarray, s: np.ndarray) -> np.ndarray:
    """REF_Q8_ROW -> float64 values."""
    return q.astype(np.float64) * s.astype(np.float64)[..., None]


def quantize_g64(x: np.ndarray, group_size: int = 64):
    """float [..., D] -> (uint32 [..., D/4], bf16 scales [..., D/64], bf16 biases)."""
    xf = np.asarray(x, dtype=np.float32)
    lead, d = xf.shape[:-1], xf.shape[-1]
    wq, s, b = quantize(xf.reshape(-1, d), group_size=group_size, bits=8)
    return wq.reshape(*lead, d // 4), s.reshape(*lead, d // group_size), b.reshape(*lead, d // group_size)


def dequant_g64(wq: np.ndarray, s_bits: np.ndarray, b_bits: np.ndarray, group_size: int = 64) -> np.ndarray:
    """MLX_Q8_G64 -> float64 values s * q + b (exact)."""
    q = unpack_bits(wq, 8).astype(np.float64)
    s = np.repeat(bf16_bits_to_f32(s_bits).astype(np.float64), group_size, axis=-1)
    b = np.repeat(bf16_bits_to_f32(b_bits).astype(np.float64), group_size, axis=-1)
    return q * s + b


__all__ = ["quantize_rows", "dequant_rows", "quantize_g64", "dequant_g64", "pack_bits"]


def take_rows(t: np.ndarray, start: int, nodes) -> np.ndarray:
    """A tree commit of one cache tensor [B, Hkv, cap, ...]
    (tree_verify.py:487-496 _keep_kv, kv8.py:143-148 take_rows): rows
    start + nodes move to start, start + 1, ... Returns the new tensor; the
    gather reads the old rows before any is written, as mx.take does."""
    out = np.array(t, copy=True)
    idx = np.asarray(nodes, dtype=np.int64) + start
    out[:, :, start:start + len(idx)] = np.take(np.asarray(t), idx, axis=2)
    return out
