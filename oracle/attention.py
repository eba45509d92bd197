"""Tree-mask attention over a long KV prefix, restated on the CPU.
TEST INFRASTRUCTURE ONLY.

Semantics of mlx-tree-spec `tree_flash` (src/mlx_tree_spec/tree_flash.py:151-196,
visibility at 40-45): queries (B, Hq, T, D) attend over the first n_kv rows of
a cache (B, Hkv, cap, D) with grouped heads (query head h uses KV head
h // (Hq / Hkv)). Row gp is visible to query q iff gp < n_kv and (gp lies
before the tail or its tail bit is set in bits[q]). Scores are
scale * q . k; softmax in float64 here; output = softmax . V.

Block statistics (`stats=True`, tree_flash.py:155-157, merged as in
tree_verify.py:389-401): for any split of the keys into blocks, a block's max
score m_b and exp-sum l_b = sum exp(s - m_b) rebuild the normaliser
sum_b l_b exp(m_b - max_b m_b).
"""

from __future__ import annotations

import numpy as np

from .tree import visibility


def tree_attention(q, k, v, n_kv: int, tail: int, bits, scale: float, return_lse: bool = False):
    """float64 tree attention.

    q: [B, Hq, T, D]; k, v: [B, Hkv, >= n_kv, D] (already dequantized values);
    bits: uint64 [B, T] (or [T], shared); tail: rows at the end of the n_kv
    valid rows covered by the bits (0: all rows visible).
    Returns out [B, Hq, T, D] (and lse [B, Hq, T] if asked). A query that sees
    no key gets output 0 and lse -inf."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)[:, :, :n_kv]
    v = np.asarray(v, dtype=np.float64)[:, :, :n_kv]
    b_, hq, t, d = q.shape
    hkv = k.shape[1]
    g = hq // hkv
    bits = np.asarray(bits, dtype=np.uint64)
    if bits.ndim == 1:
        bits = np.broadcast_to(bits, (b_, t))
    out = np.zeros((b_, hq, t, d))
    lse = np.full((b_, hq, t), -np.inf)
    for bi in range(b_):
        vis = visibility(n_kv, tail, bits[bi], t) if tail else np.ones((t, n_kv), dtype=bool)
        for h in range(hq):
            kh = k[bi, h // g]
            vh = v[bi, h // g]
            s = (q[bi, h] @ kh.T) * scale
            s = np.where(vis, s, -np.inf)
            m = s.max(axis=-1, keepdims=True)
            ok = np.isfinite(m[:, 0])
            m = np.where(np.isfinite(m), m, 0.0)
            p = np.where(vis, np.exp(s - m), 0.0)
            l_ = p.sum(axis=-1, keepdims=True)
            o = (p @ vh) / np.where(l_ > 0, l_, 1.0)
            out[bi, h] = np.where(ok[:, None], o, 0.0)
            lse[bi, h] = np.where(ok, m[:, 0] + np.log(np.where(l_[:, 0] > 0, l_[:, 0], 1.0)), -np.inf)
    return (out, lse) if return_lse else out


def merge_blocks(outs, maxs, sums):
    """Merge per-block normalised outputs with their (max, exp-sum) statistics
    into one softmax (the identity of tree_verify.py:389-401).

    outs: [..., nb, D] normalised per block; maxs, sums: [..., nb]."""
    maxs = np.asarray(maxs, dtype=np.float64)
    sums = np.asarray(sums, dtype=np.float64)
    m = maxs.max(axis=-1, keepdims=True)
    w = sums * np.exp(maxs - m)
    return (np.asarray(outs, dtype=np.float64) * w[..., None]).sum(axis=-2) / w.sum(axis=-1)[..., None]


def algorithmic_bytes(b: int, t: int, hq: int, hkv: int, d: int, n_kv: int, kv_row_bytes: float) -> float:
    """Bytes one tree-attention call must move: K and V rows once, Q in, O out."""
    return b * n_kv * hkv * kv_row_bytes * 2 + 2 * b * t * hq * d * 2


def flops(b: int, t: int, hq: int, d: int, n_kv: int) -> float:
    """QK^T plus PV over every key (masked ones counted)."""
    return 4.0 * b * t * hq * n_kv * d
