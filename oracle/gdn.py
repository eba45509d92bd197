"""GatedDeltaNet over tree nodes, restated on the CPU. TEST INFRASTRUCTURE ONLY.

The hybrid model's linear-attention layers run, for each tree node, mlx-lm's
gated delta recurrence (mlx_lm.models.gated_delta.gated_delta_update, mlx-lm
>=0.31,<0.32 per the reference's pyproject; not vendored) along the node's own
root-to-node path, starting from the committed state. This module computes
exactly that definition, node by node, so it checks the walks/siblings layout
the reference and the CUDA kernels use to share work (tree_verify.py:66-121,
149-238) rather than repeating it.

  * conv_window (tree_verify.py:111-118): the causal conv (kernel 4) of node i
    reads 3 ancestors then itself, as rows of concat(conv_state (3), qkv (n));
    past the root it reaches into conv_state from its newest row backwards.
  * prep (fused_ops.py:28-104 gdn_prep): conv, bf16, silu, bf16; v as is; q and
    k per-head RMS norm (no weight, eps 1e-6), bf16, then q * (1/Dk) and
    k * Dk^-0.5, bf16; beta = bf16(sigmoid(b));
    g = exp(-exp(A_log) * bf16(softplus(bf16(a + dt_bias)))) in float32.
  * step: S <- g S; kv = S k; delta = (v - kv) beta; S <- S + delta k^T;
    out = S q (state [Hv, Dv, Dk], value head h reads key head h / (Hv/Hk)).
  * commit (fused_ops.py:157-226 gdn_commit): the state after replaying the
    accepted path, and the conv state = the last 3 rows of the last node's window.

Parity pinned by restatement only: the reference has no test of this path
and its Metal kernels cannot run here. Arithmetic in float64 with the
reference's bf16 rounding points.
"""

from __future__ import annotations

import numpy as np

from .bf16 import round_bf16


def path(parents, i: int) -> list[int]:
    out = []
    while i >= 0:
        out.append(i)
        i = int(parents[i])
    return out[::-1]


def conv_window(parents) -> np.ndarray:
    """(n, 4) int32 row indices into concat(conv_state (3 rows), qkv (n rows)), oldest first."""
    n = len(parents)
    win = np.zeros((n, 4), dtype=np.int32)
    for i in range(n):
        p = path(parents, i)
        for back in range(4):
            win[i, 3 - back] = 3 + p[-1 - back] if back < len(p) else 2 - (back - len(p))
    return win


def prep(qkv, conv_state, conv_w, a, b, a_log, dt_bias, parents, hk: int, dk: int, hv: int, dv: int):
    """qkv (n, C), conv_state (3, C), conv_w (C, 4), a/b (n, Hv) as bf16 values;
    a_log, dt_bias (Hv,) float. Returns q, k (n, Hk, Dk), v (n, Hv, Dv), beta
    (n, Hv) as bf16 values and g (n, Hv) float32."""
    n = qkv.shape[0]
    src = np.concatenate([np.asarray(conv_state, np.float64), np.asarray(qkv, np.float64)], axis=0)
    win = conv_window(parents)
    w = np.asarray(conv_w, np.float64)
    acc = sum(src[win[:, j]] * w[:, j] for j in range(4))
    cv = round_bf16(acc).astype(np.float64)
    s = round_bf16(cv / (1.0 + np.exp(-cv))).astype(np.float64)
    qk = hk * dk

    def norm(x):
        inv = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + 1e-6)
        return round_bf16(x * inv).astype(np.float64)

    q = round_bf16(norm(s[:, :qk].reshape(n, hk, dk)) / dk)
    k = round_bf16(norm(s[:, qk:2 * qk].reshape(n, hk, dk)) * dk ** -0.5)
    v = s[:, 2 * qk:2 * qk + hv * dv].reshape(n, hv, dv).astype(np.float32)
    ab = round_bf16(np.asarray(a, np.float64) + np.asarray(dt_bias, np.float64)[None]).astype(np.float64)
    sp = np.where(ab > 20.0, ab, np.log1p(np.exp(np.minimum(ab, 20.0))))
    g = np.exp(-np.exp(np.asarray(a_log, np.float64))[None] * round_bf16(sp)).astype(np.float32)
    beta = round_bf16(1.0 / (1.0 + np.exp(-np.asarray(b, np.float64))))
    return q, k, v, g, beta


def _step(S, q, k, v, g, beta, rep: int):
    """One recurrence step for all value heads; returns (new state, output)."""
    kk = np.repeat(np.asarray(k, np.float64), rep, axis=0)   # (Hv, Dk)
    qq = np.repeat(np.asarray(q, np.float64), rep, axis=0)
    S = S * np.asarray(g, np.float64)[:, None, None]
    kv = np.einsum("hvk,hk->hv", S, kk)
    delta = (np.asarray(v, np.float64) - kv) * np.asarray(beta, np.float64)[:, None]
    S = S + delta[:, :, None] * kk[:, None, :]
    return S, np.einsum("hvk,hk->hv", S, qq)


def tree_recurrence(q, k, v, g, beta, state0, parents) -> np.ndarray:
    """y (n, Hv, Dv) float64: each node's output along its root path from state0
    (Hv, Dv, Dk). Parents come before children, so each node steps from its
    parent's state."""
    n, hv = v.shape[0], v.shape[1]
    rep = hv // q.shape[1]
    states = [None] * n
    y = np.zeros(v.shape, dtype=np.float64)
    for i in range(n):
        p = int(parents[i])
        S0 = np.asarray(state0, np.float64) if p < 0 else states[p]
        states[i], y[i] = _step(S0, q[i], k[i], v[i], g[i], beta[i], rep)
    return y


def commit(k, v, g, beta, state0, conv_state, qkv, parents, nodes):
    """(state (Hv, Dv, Dk) float64, conv_state (3, C)) after the accepted path `nodes`."""
    rep = v.shape[1] // k.shape[1]
    S = np.asarray(state0, np.float64)
    for t in nodes:
        S, _ = _step(S, k[t], k[t], v[t], g[t], beta[t], rep)
    src = np.concatenate([np.asarray(conv_state), np.asarray(qkv)], axis=0)
    return S, src[conv_window(parents)[nodes[-1], 1:]]
