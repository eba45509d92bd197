"""MLX affine-quantized weights and the quantized matmul, restated on the CPU.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Format (MLX `mx.quantize(w, group_size=64, bits=4)`, as consumed by the
reference; mlx-tree-spec src/mlx_tree_spec/qmm_packed.py:115,200-201,348-349,
635-636 and packed_linear.py:72-80):
  * w: uint32 [N, K*bits/32]. Word c of row n holds elements 32c/bits ..
    32c/bits + 32/bits - 1 of that row; element i of the word sits in bits
    bits*i .. bits*i + bits - 1 (lowest bits first), i.e. for 4 bits
    `(word >> (4*i)) & 0xF` is element 8c + i.
  * scales, biases: bf16 [N, K/group_size]; element value = s * q + b.

Dequantization rule (bit-exact contract of the B200 build): the reference's
kernels compute `T(float(q) * float(s) + float(b))` (qmm_packed.py:200,348,635),
i.e. an fp32 multiply-add rounded to bf16. The build fixes this as
`bf16_rne(fp32_fma(q, s, b))`: the exact value q*s + b is rounded once to
float32, then to bf16 (round to nearest even both times).

Quantizer: MLX's `mx.quantize` (mlx 0.32.2, not vendored) is min/max affine
per group; its exact edge rules are not pinned by the reference. The build's
own quantizer below (documented, deterministic) produces test weights; parity
is defined on the stored (w, scales, biases), which the oracle and the GPU
consume identically.
"""

from __future__ import annotations

import numpy as np

from .bf16 import bf16_bits_to_f32, f32_to_bf16_bits


def pack_bits(q: np.ndarray, bits: int) -> np.ndarray:
    """Integer codes [..., K] (0 <= q < 2**bits) -> uint32 words [..., K*bits/32].

    Element i of each word occupies bits bits*i .. (lowest first), as MLX
    stores it (qmm_packed.py:115)."""
    per = 32 // bits
    q = np.asarray(q).astype(np.uint32)
    assert q.shape[-1] % per == 0
    q = q.reshape(*q.shape[:-1], q.shape[-1] // per, per)
    shifts = (np.arange(per, dtype=np.uint32) * bits).astype(np.uint32)
    return np.bitwise_or.reduce(q << shifts, axis=-1).astype(np.uint32)


def unpack_bits(w: np.ndarray, bits: int) -> np.ndarray:
    """uint32 words [..., W] -> integer codes [..., W*32/bits] (uint8)."""
    per = 32 // bits
    w = np.asarray(w, dtype=np.uint32)
    shifts = (np.arange(per, dtype=np.uint32) * bits).astype(np.uint32)
    q = (w[..., None] >> shifts) & np.uint32((1 << bits) - 1)
    return q.reshape(*w.shape[:-1], w.shape[-1] * per).astype(np.uint8)


def quantize(w: np.ndarray, group_size: int = 64, bits: int = 4):
    """float [N, K] -> (wq uint32 [N, K*bits/32], scales bf16 bits, biases bf16 bits).

    Per group of `group_size` along K: bias = min, scale = (max - min) /
    (2**bits - 1), both rounded to bf16; q = clip(rint((w - b) / s)) against
    the rounded scale and bias. A constant group gets scale 0 and q = 0."""
    w = np.asarray(w, dtype=np.float32)
    n, k = w.shape
    assert k % group_size == 0
    levels = (1 << bits) - 1
    g = w.reshape(n, k // group_size, group_size)
    wmin = g.min(axis=-1)
    wmax = g.max(axis=-1)
    s_bits = f32_to_bf16_bits((wmax - wmin) / np.float32(levels))
    b_bits = f32_to_bf16_bits(wmin)
    s = bf16_bits_to_f32(s_bits)[..., None]
    b = bf16_bits_to_f32(b_bits)[..., None]
    safe = np.where(s == 0, np.float32(1), s)
    q = np.where(s == 0, 0, np.clip(np.rint((g - b) / safe), 0, levels))
    q = q.reshape(n, k).astype(np.uint8)
    return pack_bits(q, bits), s_bits, b_bits


def _fma_to_f32(a: np.ndarray, b: np.ndarray, c: np.ndarray) -> np.ndarray:
    """Correctly rounded float32 of a*b + c for float32-representable inputs.

    a*b is exact in float64 (24 + 24 < 53 bits). The float64 sum is made
    round-to-odd with a TwoSum error term, after which rounding to float32 is
    the single correctly rounded result (53 >= 24 + 2), i.e. fmaf()."""
    p = a.astype(np.float64) * b.astype(np.float64)
    c = c.astype(np.float64)
    s = p + c
    bb = s - p
    err = (p - (s - bb)) + (c - bb)
    inexact = err != 0
    if inexact.any():
        bits = s.view(np.uint64)
        even = (bits & np.uint64(1)) == 0
        fix = inexact & even & np.isfinite(s)
        if fix.any():
            toward = np.where(err > 0, np.inf, -np.inf)
            s = s.copy()
            s[fix] = np.nextafter(s[fix], toward[fix])
    return s.astype(np.float32)


def dequantize(wq, scales_bits, biases_bits, group_size: int = 64, bits: int = 4) -> np.ndarray:
    """(wq, scales, biases) -> bf16 bits [N, K] by the rule bf16(fp32_fma(q, s, b))."""
    q = unpack_bits(wq, bits).astype(np.float32)
    n, k = q.shape
    s = np.repeat(bf16_bits_to_f32(scales_bits), group_size, axis=-1).reshape(n, k)
    b = np.repeat(bf16_bits_to_f32(biases_bits), group_size, axis=-1).reshape(n, k)
    return f32_to_bf16_bits(_fma_to_f32(q, s, b))


def qmm(x_bits, wq, scales_bits, biases_bits, group_size: int = 64, bits: int = 4) -> np.ndarray:
    """y = x @ dequantize(w).T in float64 (the `exact` of the reference's
    tests/test_units.py:108: x in float32 times the dequantized weight).

    x_bits: bf16 bits [M, K]. Returns float64 [M, N]."""
    x = bf16_bits_to_f32(x_bits).astype(np.float64)
    w = bf16_bits_to_f32(dequantize(wq, scales_bits, biases_bits, group_size, bits)).astype(np.float64)
    return x @ w.T


def qmm_f32(x_f32: np.ndarray, w_deq_f32: np.ndarray) -> np.ndarray:
    """The CPU baseline's arithmetic: float32 matmul on a pre-dequantized weight
    (the torch-CPU/numpy fp32 fallback of the reference's operator)."""
    return x_f32 @ w_deq_f32.T


def algorithmic_bytes(m: int, n: int, k: int, group_size: int = 64) -> int:
    """Bytes one quantized matmul must move: codes + scales/biases + x + y."""
    return n * k // 2 + n * (k // group_size) * 4 + m * k * 2 + m * n * 2


def dequantize_fast_f32(wq, scales_bits, biases_bits, group_size: int = 64) -> np.ndarray:
    """Same values as dequantize() (as float32), computed in float32 for speed.

    For 4-bit codes q*s is exact in float32 (4 + 8 significant bits), so one
    float32 add gives fmaf(q, s, b); the bf16 rounding is then done on the
    bits. Used by the CPU baseline timing, where the float64 path is too slow."""
    q = unpack_bits(wq, 4).astype(np.float32)
    n, k = q.shape
    g = k // group_size
    s = bf16_bits_to_f32(scales_bits).reshape(n, g, 1)
    b = bf16_bits_to_f32(biases_bits).reshape(n, g, 1)
    f = (q.reshape(n, g, group_size) * s + b).reshape(n, k)
    u = f.view(np.uint32)
    r = (u + (((u >> 16) & 1) + 0x7FFF)) & np.uint32(0xFFFF0000)
    return r.view(np.float32)


def qmm_cpu(x_bits, wq, scales_bits, biases_bits, threads: int = 1) -> np.ndarray:
    """The CPU port of the operator (timed as the CPU baseline): dequantize the
    packed weight to bf16 values, then a float32 matmul, row blocks of the
    weight spread over `threads` host threads."""
    from concurrent.futures import ThreadPoolExecutor

    x = bf16_bits_to_f32(x_bits)
    n = wq.shape[0]
    blocks = max(1, threads)
    edges = [n * i // blocks for i in range(blocks + 1)]

    def part(i):
        a, b_ = edges[i], edges[i + 1]
        w = dequantize_fast_f32(wq[a:b_], scales_bits[a:b_], biases_bits[a:b_])
        return x @ w.T

    if blocks == 1:
        return part(0)
    with ThreadPoolExecutor(blocks) as ex:
        return np.concatenate(list(ex.map(part, range(blocks))), axis=1)
