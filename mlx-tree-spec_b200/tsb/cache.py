"""KV-cache containers with the layout the reference's caches have.

Fields mirror mlx-lm's KVCache as the reference reads it (keys/values
(B, Hkv, capacity, D), `offset` valid rows; mlx-tree-spec
src/mlx_tree_spec/tree_flash.py:162-168) and the reference's Q8KVCache
(int8 rows + float32 scale per row in k_scale/v_scale; kv8.py:95-148). The
MLX 8-bit g64 cache (mlx-lm's quantized cache) stores uint32 words of four
codes plus bf16 scales/biases per 64 values.

These are plain holders of device tensors: filling them (append, quantize on
append) is the caller's business here.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ._lib import TSB_KV_BF16, TSB_KV_MLX_Q8_G64, TSB_KV_REF_Q8_ROW


@dataclass
class KVCache:
    keys: torch.Tensor      # bf16 (B, Hkv, cap, D)
    values: torch.Tensor
    offset: int
    kv_format: int = TSB_KV_BF16


@dataclass
class Q8KVCache:
    keys: torch.Tensor      # int8 (B, Hkv, cap, D)
    values: torch.Tensor
    k_scale: torch.Tensor   # float32 (B, Hkv, cap)
    v_scale: torch.Tensor
    offset: int
    kv_format: int = TSB_KV_REF_Q8_ROW


@dataclass
class MLXQ8KVCache:
    keys: torch.Tensor      # uint32 words as int32 (B, Hkv, cap, D/4)
    values: torch.Tensor
    k_scales: torch.Tensor  # bf16 (B, Hkv, cap, D/64)
    k_biases: torch.Tensor
    v_scales: torch.Tensor
    v_biases: torch.Tensor
    offset: int
    kv_format: int = TSB_KV_MLX_Q8_G64
