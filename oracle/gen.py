"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations. TEST INFRASTRUCTURE ONLY.

RNG: numpy.random.default_rng(seed). Config 1 uses seed 0; sweeps use
1000 + config index. x ~ N(0, 1) -> bf16; W ~ N(0, 0.02) -> 4-bit g64;
K/V and Q ~ N(0, 1) -> bf16. Tree parents: parent[0] = -1, parent[i] ~
U{-1 .. i-1}, redrawn while the node's depth would exceed 8.
"""

from __future__ import annotations

import numpy as np

from .bf16 import f32_to_bf16_bits
from .qmm import quantize

QMM_SHAPES = ((6144, 5120), (34816, 5120), (5120, 17408))
QMM_SWEEP_M = (1, 8, 16, 32, 64, 128)
PREFILL_M = 4096
ATTN = dict(T=32, Hq=24, Hkv=4, D=256, L=(1024, 8192, 32768), B=(1, 4))


def x_bf16(rng, m: int, k: int, std: float = 1.0) -> np.ndarray:
    return f32_to_bf16_bits(rng.standard_normal((m, k), dtype=np.float32) * np.float32(std))


def weights_w4g64(rng, n: int, k: int, std: float = 0.02):
    w = rng.standard_normal((n, k), dtype=np.float32) * np.float32(std)
    return quantize(w, group_size=64, bits=4)


def config1():
    """Config 1: x bf16 [16, 5120] ~ N(0,1); W [6144, 5120] ~ N(0, 0.02) -> 4-bit g64; seed 0."""
    rng = np.random.default_rng(0)
    x = x_bf16(rng, 16, 5120)
    wq, s, b = weights_w4g64(rng, 6144, 5120)
    return x, wq, s, b


def tree_parents(rng, t: int, max_depth: int = 8) -> np.ndarray:
    """parent[0] = -1; parent[i] ~ U{-1..i-1}, redrawn while depth > max_depth."""
    parents = np.full(t, -1, dtype=np.int32)
    depth = np.zeros(t, dtype=np.int32)
    for i in range(1, t):
        while True:
            p = int(rng.integers(-1, i))
            d = 0 if p < 0 else depth[p] + 1
            if d <= max_depth:
                break
        parents[i] = p
        depth[i] = d
    return parents


def chain_parents(t: int) -> np.ndarray:
    return np.arange(-1, t - 1, dtype=np.int32)
