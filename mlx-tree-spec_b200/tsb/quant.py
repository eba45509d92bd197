"""Weight/KV quantizers for producing inputs (not on the hot path).

`quantize` is this library's documented stand-in for MLX's `mx.quantize`
(min/max affine per group, scale and bias rounded to bf16, codes against the
rounded values); mlx-tree-spec consumes MLX-format (w, scales, biases) as
given (src/mlx_tree_spec/packed_linear.py:136-156), so any quantizer's output
is a valid input. `quantize_rows` is the reference's 8-bit KV row quantizer
(kv8.py:39-43). Both run as torch tensor ops on whatever device the input is
on; they only make test and benchmark inputs.
"""

from __future__ import annotations

import torch


def pack_bits(q: torch.Tensor, bits: int) -> torch.Tensor:
    """Codes (..., K) -> int32 words (..., K*bits/32), element i of a word in
    bits bits*i.. (lowest first): MLX's layout."""
    per = 32 // bits
    q = q.to(torch.int64).reshape(*q.shape[:-1], q.shape[-1] // per, per)
    shifts = torch.arange(per, device=q.device, dtype=torch.int64) * bits
    words = (q << shifts).sum(dim=-1)
    words = torch.where(words >= 2**31, words - 2**32, words)
    return words.to(torch.int32)


def unpack_bits(w: torch.Tensor, bits: int) -> torch.Tensor:
    per = 32 // bits
    w64 = w.to(torch.int64) & 0xFFFFFFFF
    shifts = torch.arange(per, device=w.device, dtype=torch.int64) * bits
    q = (w64[..., None] >> shifts) & ((1 << bits) - 1)
    return q.reshape(*w.shape[:-1], w.shape[-1] * per).to(torch.uint8)


def quantize(w: torch.Tensor, group_size: int = 64, bits: int = 4):
    """float (N, K) -> (w int32 (N, K*bits/32), scales bf16 (N, G), biases bf16 (N, G))."""
    n, k = w.shape
    levels = (1 << bits) - 1
    g = w.to(torch.float32).reshape(n, k // group_size, group_size)
    wmin = g.amin(dim=-1)
    wmax = g.amax(dim=-1)
    s = ((wmax - wmin) / levels).to(torch.bfloat16)
    b = wmin.to(torch.bfloat16)
    sf = s.to(torch.float32)[..., None]
    bf = b.to(torch.float32)[..., None]
    safe = torch.where(sf == 0, torch.ones_like(sf), sf)
    q = torch.where(sf == 0, torch.zeros_like(g), torch.clamp(torch.round((g - bf) / safe), 0, levels))
    return pack_bits(q.reshape(n, k), bits), s, b


def quantize_rows(x: torch.Tensor):
    """(..., D) -> int8 rows and float32 scales (...), as kv8.quantize_rows."""
    xf = x.to(torch.float32)
    s = torch.clamp(xf.abs().amax(dim=-1, keepdim=True) / 127.0, min=1e-6)
    q = torch.clamp(torch.round(xf / s), -127, 127).to(torch.int8)
    return q, s[..., 0]


def quantize_g64(x: torch.Tensor, group_size: int = 64):
    """(..., D) -> MLX 8-bit g64: int32 words (..., D/4), bf16 scales/biases (..., D/64)."""
    lead, d = x.shape[:-1], x.shape[-1]
    w, s, b = quantize(x.reshape(-1, d), group_size=group_size, bits=8)
    return w.reshape(*lead, d // 4), s.reshape(*lead, d // group_size), b.reshape(*lead, d // group_size)
