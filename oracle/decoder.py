"""The verify-step decoder layer (the gated-q layer), restated on the CPU.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Follows mlx-tree-spec's gated-q layer and layer loop:
  * batch_forward (src/mlx_tree_spec/tree_verify.py:414-447): x = input norm of
    h; per layer r = attention(x); h, x = add_rms_norm(h, r, post norm);
    h, x = add_rms_norm(h, mlp(x), next layer's input norm (or the final norm)).
  * batch_attention / _attn_core (tree_verify.py:311-367): q_proj output split
    per head into queries and gate (318-319), k_norm(k_proj(x)), v_proj(x),
    q_norm(queries), rope of queries and keys at each node's position
    (depth + prefix length, 422 and 342-348), keys/values appended to the
    cache, tree attention (scale D^-0.5), o_proj(out * sigmoid(gate)) (327).
  * add_rms_norm (fused_ops.py:107-129): h = T(x + r),
    n = T(w * T(h * rsqrt(mean(h^2) + eps))); nn.RMSNorm (mx.fast.rms_norm)
    rounds the same way without the residual.
  * rope: mx.fast.rope, non-traditional (mlx 0.32.2, not vendored): for
    i < dims/2 the pair (x_i, x_{i+dims/2}) turns by
    angle = pos * scale * base^(-2i/dims); dims beyond `dims` pass through.
  * MLP: down(silu(gate(x)) * up(x)), silu(g) = g * sigmoid(g), each op
    rounded to bf16 (mlx-lm SwiGLU).
Every op's output is rounded to bf16 where the reference materialises a bf16
tensor; inside an op the arithmetic is float64. The quantized projections use
oracle.qmm (dequantize, float64 matmul) and attention oracle.attention.
"""

from __future__ import annotations

import numpy as np

from . import attention, kv, qmm, tree
from .bf16 import bf16_bits_to_f32, f32_to_bf16_bits, round_bf16


def rms_norm(x, w, eps: float, r=None):
    """(h, n): h = bf16(x + r) (x when r is None), n = bf16(w * bf16(h * inv))."""
    x = np.asarray(x, dtype=np.float32)
    h = round_bf16(x.astype(np.float64) + np.asarray(r, np.float64)) if r is not None else x
    inv = 1.0 / np.sqrt(np.mean(h.astype(np.float64) ** 2, axis=-1, keepdims=True) + eps)
    n = round_bf16(np.asarray(w, np.float64) * round_bf16(h.astype(np.float64) * inv))
    return h, n


def rope(x, pos, dims: int, base: float, scale: float = 1.0):
    """mx.fast.rope (non-traditional) of rows x [..., D] at positions pos [...]."""
    x = np.asarray(x, dtype=np.float64)
    half = dims // 2
    j = np.arange(half, dtype=np.float64)
    inv_freq = base ** (-j / half)
    ang = np.asarray(pos, np.float64)[..., None] * scale * inv_freq
    c, s = np.cos(ang), np.sin(ang)
    out = x.copy()
    x1, x2 = x[..., :half], x[..., half:dims]
    out[..., :half] = x1 * c - x2 * s
    out[..., half:dims] = x1 * s + x2 * c
    return round_bf16(out)


def sigmoid_bf16(g):
    return round_bf16(1.0 / (1.0 + np.exp(-np.asarray(g, np.float64))))


def qkv_prep(qkv, hq: int, hkv: int, q_norm, k_norm, eps: float, positions, b: int, t: int, rope_dims: int,
             rope_base: float, rope_scale: float = 1.0, d: int = 256):
    """qkv [B*T, >= (2 hq + 2 hkv) d] (bf16 values) -> queries [B, hq, T, d],
    keys and values [B, hkv, T, d] (after norm and rope), gate [B*T, hq, d]."""
    m = b * t
    qg = qkv[:, :hq * 2 * d].reshape(m, hq, 2 * d)
    q, gate = qg[..., :d], qg[..., d:]
    k = qkv[:, hq * 2 * d:hq * 2 * d + hkv * d].reshape(m, hkv, d)
    v = qkv[:, hq * 2 * d + hkv * d:hq * 2 * d + 2 * hkv * d].reshape(m, hkv, d)
    _, qn = rms_norm(q, q_norm, eps)
    _, kn = rms_norm(k, k_norm, eps)
    pos = np.asarray(positions).reshape(m, 1)
    qr = rope(qn, pos, rope_dims, rope_base, rope_scale)
    kr = rope(kn, pos, rope_dims, rope_base, rope_scale)
    to_bhtd = lambda a, h: a.reshape(b, t, h, d).transpose(0, 2, 1, 3)  # noqa: E731
    return to_bhtd(qr, hq), to_bhtd(kr, hkv), to_bhtd(np.asarray(v, np.float32), hkv), gate


def attn_gate(out_bhtd, gate):
    """o_proj input [B*T, hq*d] = bf16(out * bf16(sigmoid(gate)))."""
    b, h, t, d = out_bhtd.shape
    o = np.asarray(out_bhtd, np.float64).transpose(0, 2, 1, 3).reshape(b * t, h, d)
    return round_bf16(o * sigmoid_bf16(gate)).reshape(b * t, h * d)


def swiglu(gu):
    """[M, 2I] = [g | u] -> bf16(bf16(g * bf16(sigmoid(g))) * u)."""
    i = gu.shape[-1] // 2
    g, u = np.asarray(gu[..., :i], np.float64), np.asarray(gu[..., i:], np.float64)
    return round_bf16(round_bf16(g * sigmoid_bf16(g)) * u)


def linear(x, w):
    """A 4-bit g64 projection: bf16(x @ dequant(w).T); x as bf16 values, w = (wq, s_bits, b_bits)."""
    return round_bf16(qmm.qmm(f32_to_bf16_bits(np.asarray(x, np.float32)), *w))


def _stored(rows, kv_format):
    """The values a cache of this format holds for appended rows."""
    if kv_format == "mlx_q8":
        return kv.dequant_g64(*kv.quantize_g64(rows))
    if kv_format == "ref_q8":
        return kv.dequant_rows(*kv.quantize_rows(rows))
    return rows


def layer_step(h, x, p, k_cache, v_cache, parents, offsets, cfg, next_norm, kv_format: str = "bf16"):
    """One decoder layer on the nodes. h, x [B*T, hidden] (bf16 values);
    k_cache/v_cache float [B, hkv, cap, d] (the prefix in rows < offsets[b],
    updated in place with the nodes' rows, as a cache of `kv_format` stores
    them); p: the layer's weights. Returns the new (h, x)."""
    b, t = parents.shape
    hq, hkv, d, eps = cfg["hq"], cfg["hkv"], cfg["d"], cfg["eps"]
    depth = np.stack([tree.depth(parents[i]) for i in range(b)])
    positions = (depth + np.asarray(offsets)[:, None]).reshape(-1)
    qkv_out = linear(x, p["qkv"])
    q, k, v, gate = qkv_prep(qkv_out, hq, hkv, p["q_norm"], p["k_norm"], eps, positions, b, t, cfg["rope_dims"],
                             cfg["rope_base"])
    bits = np.stack([tree.ancestor_bits_u64(parents[i]) for i in range(b)])
    outs = []
    for i in range(b):
        off = int(offsets[i])
        k_cache[i, :, off:off + t] = _stored(k[i], kv_format)
        v_cache[i, :, off:off + t] = _stored(v[i], kv_format)
        o = attention.tree_attention(q[i:i + 1], k_cache[i:i + 1], v_cache[i:i + 1], off + t, t, bits[i:i + 1],
                                     d ** -0.5)
        outs.append(round_bf16(o))
    o = np.concatenate(outs, axis=0)
    r = linear(attn_gate(o, gate), p["o"])
    h, x = rms_norm(h, p["post_norm"], eps, r)
    r = linear(swiglu(linear(x, p["gate_up"])), p["down"])
    return rms_norm(h, next_norm, eps, r)


__all__ = ["rms_norm", "rope", "qkv_prep", "attn_gate", "swiglu", "linear", "layer_step",
           "bf16_bits_to_f32", "kv"]
