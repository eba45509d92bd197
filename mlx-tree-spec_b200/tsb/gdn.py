"""GatedDeltaNet over tree nodes on the GPU: the linear-attention layers of the
hybrid model's verify pass.

Mirrors, over torch CUDA tensors:
  walks(parents)            the walk fields of tree_verify.Tree
                            (mlx-tree-spec src/mlx_tree_spec/tree_verify.py:66-121:
                            rows, sibs, owner, lmax, conv_idx)
  gdn_prep(...)             fused_ops.gdn_prep (fused_ops.py:92-104)
  tree_gated_delta(...)     tree_verify.tree_gated_delta (tree_verify.py:225-238)
  gdn_commit(rec, ...)      fused_ops.gdn_commit (fused_ops.py:213-226)

Walks: every leaf's root-to-leaf path is a candidate walk. A leaf whose parent
another walk passes through (and continues past) rides on that walk as a side
step at its depth, computed from the walk's state before that step: it costs
no state read of its own. Each node's output is written by the first walk that
holds it (owner). The walk layout only decides who computes what; every
node's output is the recurrence along its own root path either way.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from functools import lru_cache

import numpy as np
import torch

from . import _lib
from ._lib import check


@dataclass(frozen=True)
class Walks:
    rows: tuple          # each walk's node path (root first)
    sibs: tuple          # per walk and step: the side leaf at that step or -1
    owner: tuple         # per node: the walk that writes its output
    lmax: int
    conv_idx: np.ndarray  # (n, 4) int32 rows of concat(conv_state, qkv), oldest first


def _check_parents(parents) -> tuple:
    """parents: a sequence of parent indices, or a tree object carrying them in
    `.parents` (as the reference's Tree does)."""
    parents = getattr(parents, "parents", parents)
    p = tuple(int(x) for x in parents)
    if not p or p[0] != -1 or any(not 0 <= q < i for i, q in enumerate(p) if i):
        raise ValueError("parents: node 0 is the root (-1) and every other parent precedes its node")
    return p


@lru_cache(maxsize=256)
def _walks(parents: tuple) -> Walks:
    n = len(parents)
    has_child = [False] * n
    for i in range(1, n):
        has_child[parents[i]] = True

    def root_path(i):
        out = []
        while i >= 0:
            out.append(i)
            i = parents[i]
        return out[::-1]

    rows, sibs = [], []
    for leaf in (i for i in range(n) if not has_child[i]):
        p = root_path(leaf)
        t = len(p) - 1          # the leaf's step
        host = None
        if t >= 1:
            for r, rp in enumerate(rows):
                if len(rp) > t and rp[t - 1] == p[t - 1] and sibs[r][t] < 0:
                    host = r
                    break
        if host is None:
            rows.append(p)
            sibs.append([-1] * len(p))
        else:
            sibs[host][t] = leaf
    owner = [-1] * n
    for r, (rp, rs) in enumerate(zip(rows, sibs)):
        for i in rp + [x for x in rs if x >= 0]:
            if owner[i] < 0:
                owner[i] = r
    conv = np.zeros((n, 4), dtype=np.int32)
    for i in range(n):
        p = root_path(i)
        for back in range(4):
            conv[i, 3 - back] = 3 + p[-1 - back] if back < len(p) else 2 - (back - len(p))
    return Walks(tuple(tuple(r) for r in rows), tuple(tuple(s) for s in sibs), tuple(owner),
                 max(len(r) for r in rows), conv)


def walks(parents) -> Walks:
    """The walk layout of a tree given each node's parent (node 0 the root)."""
    return _walks(_check_parents(parents))


_DEV: dict = {}


def _device_walks(parents, device):
    """(paths, sibs, owner, conv_idx) int32 device tensors of a tree, cached per tree and device."""
    p = _check_parents(parents)
    key = (p, str(device))
    hit = _DEV.get(key)
    if hit is None:
        w = _walks(p)
        pad = lambda rs: [list(r) + [-1] * (w.lmax - len(r)) for r in rs]  # noqa: E731
        hit = tuple(torch.tensor(np.asarray(x, dtype=np.int32), device=device)
                    for x in (pad(w.rows), pad(w.sibs), list(w.owner), w.conv_idx))
        if len(_DEV) > 256:
            _DEV.clear()
        _DEV[key] = hit
    return hit


def _st(t):
    return torch.cuda.current_stream(t.device).cuda_stream


def _p(t):
    return t.data_ptr()


def _need(*ts):
    for t in ts:
        if not t.is_cuda or not t.is_contiguous():
            raise ValueError("tsb.gdn takes contiguous CUDA tensors (there is no CPU path)")


def _expect(t, numel: int, dtype, name: str):
    """The kernels index by the head counts, so every buffer's size and dtype is checked here."""
    if t.dtype != dtype or t.numel() != numel:
        raise ValueError(f"{name}: want {numel} elements of {dtype}, got {tuple(t.shape)} {t.dtype}")


def conv_idx(parents, device) -> torch.Tensor:
    """walks(parents).conv_idx as an (n*4,) int32 device tensor (cached)."""
    return _device_walks(parents, device)[3].view(-1)


def gdn_prep(qkv, conv_state, conv_idx, conv_w, a, b, A_log, dt_bias, hk: int, dk: int, hv: int, dv: int):
    """(q, k, v, g, beta) for every node, as gdn_prep returns them: q, k
    (1, n, Hk, Dk), v (1, n, Hv, Dv), beta (1, n, Hv) bf16; g (1, n, Hv) float32.
    qkv (1, n, C) bf16; conv_state (1, 3, C); conv_idx (n*4,) or (n, 4) int32
    (walks(parents).conv_idx on the device); conv_w (C, 4); a, b (1, n, Hv);
    A_log, dt_bias (Hv,) (any float dtype: read as float32)."""
    n = qkv.shape[-2]
    dev = qkv.device
    qkv, conv_state, conv_w, a, b = (t.contiguous() for t in (qkv, conv_state, conv_w, a, b))
    ci = conv_idx.to(device=dev, dtype=torch.int32).contiguous()
    alog = A_log.to(device=dev, dtype=torch.float32).contiguous()
    dtb = dt_bias.to(device=dev, dtype=torch.float32).contiguous()
    _need(qkv, conv_state, conv_w, a, b)
    c = hk * dk * 2 + hv * dv
    bf = torch.bfloat16
    for t, numel, dt, name in ((qkv, n * c, bf, "qkv"), (conv_state, 3 * c, bf, "conv_state"),
                               (conv_w, 4 * c, bf, "conv_w"), (a, n * hv, bf, "a"), (b, n * hv, bf, "b"),
                               (ci, 4 * n, torch.int32, "conv_idx"), (alog, hv, torch.float32, "A_log"),
                               (dtb, hv, torch.float32, "dt_bias")):
        _expect(t, numel, dt, name)
    e = lambda *s, dt=torch.bfloat16: torch.empty(*s, dtype=dt, device=dev)  # noqa: E731
    q, k, v, g, beta = e(1, n, hk, dk), e(1, n, hk, dk), e(1, n, hv, dv), e(1, n, hv, dt=torch.float32), e(1, n, hv)
    lib = _lib.load()
    st = lib.tsb_gdn_prep(_p(qkv), _p(conv_state), _p(ci), _p(conv_w), _p(a), _p(b), _p(alog), _p(dtb), _p(q), _p(k),
                          _p(v), _p(g), _p(beta), n, hk, dk, hv, dv, _st(qkv))
    if check(st, "tsb_gdn_prep") == _lib.TSB_EUNSUPPORTED:
        raise ValueError(f"gdn_prep: unsupported heads (Hk={hk}, Dk={dk}, Hv={hv}, Dv={dv})")
    return q, k, v, g, beta


def tree_gated_delta(q, k, v, g, beta, state, parents):
    """Outputs (1, n, Hv, Dv) bf16 of the gated delta recurrence for every node,
    each along its own root path from `state` (1, Hv, Dv, Dk) float32 (not
    modified). q, k (1, n, Hk, Dk); v (1, n, Hv, Dv); g (float32), beta (1, n, Hv)."""
    _, n, hk, dk = k.shape
    hv, dv = v.shape[2:]
    paths, sibs, owner, _ = _device_walks(parents, q.device)
    if len(owner) != n:
        raise ValueError(f"tree of {len(owner)} nodes for {n} nodes of inputs")
    _need(q, k, v, g, beta, state)
    bf = torch.bfloat16
    for t, numel, dt, name in ((q, n * hk * dk, bf, "q"), (k, n * hk * dk, bf, "k"), (v, n * hv * dv, bf, "v"),
                               (g, n * hv, torch.float32, "g"), (beta, n * hv, bf, "beta"),
                               (state, hv * dv * dk, torch.float32, "state")):
        _expect(t, numel, dt, name)
    y = torch.empty((1, n, hv, dv), dtype=torch.bfloat16, device=q.device)
    lib = _lib.load()
    st = lib.tsb_tree_gated_delta(_p(q), _p(k), _p(v), _p(g), _p(beta), _p(state), _p(paths), _p(sibs), _p(owner),
                                  paths.shape[0], paths.shape[1], n, hk, dk, hv, dv, _p(y), _st(q))
    if check(st, "tsb_tree_gated_delta") == _lib.TSB_EUNSUPPORTED:
        raise ValueError(f"tree_gated_delta: unsupported heads (Hk={hk}, Dk={dk}, Hv={hv}, Dv={dv})")
    return y


def gdn_commit(rec, parents, nodes):
    """New [conv_state (1, 3, C), state (1, Hv, Dv, Dk)] after the accepted
    `nodes` of a tree pass, from what the pass recorded:
    rec = (conv_state, state0, qkv, q, k, v, g, beta)."""
    conv_state, state0, qkv, _, k, v, g, beta = rec
    _, n, hk, dk = k.shape
    hv, dv = v.shape[2:]
    nodes = [int(i) for i in nodes]
    if not nodes:
        raise ValueError("gdn_commit: empty path")
    _need(conv_state, state0, qkv, k, v, g, beta)
    c = hk * dk * 2 + hv * dv
    bf = torch.bfloat16
    for t, numel, dt, name in ((k, n * hk * dk, bf, "k"), (v, n * hv * dv, bf, "v"), (g, n * hv, torch.float32, "g"),
                               (beta, n * hv, bf, "beta"), (state0, hv * dv * dk, torch.float32, "state0"),
                               (conv_state, 3 * c, bf, "conv_state"), (qkv, n * c, bf, "qkv")):
        _expect(t, numel, dt, name)
    _, _, owner, cidx = _device_walks(parents, k.device)
    if len(owner) != n:
        raise ValueError(f"tree of {len(owner)} nodes for {n} nodes of inputs")
    state = torch.empty_like(state0)
    conv = torch.empty_like(conv_state)
    lib = _lib.load()
    arr = (ctypes.c_int32 * len(nodes))(*nodes)
    st = lib.tsb_gdn_commit(_p(k), _p(v), _p(g), _p(beta), _p(state0), _p(conv_state), _p(qkv), _p(cidx), arr,
                            len(nodes), n, hk, dk, hv, dv, _p(state), _p(conv), _st(k))
    if check(st, "tsb_gdn_commit") == _lib.TSB_EUNSUPPORTED:
        raise ValueError(f"gdn_commit: unsupported (Hv={hv}, path of {len(nodes)})")
    return [conv, state]


__all__ = ["Walks", "walks", "conv_idx", "gdn_prep", "tree_gated_delta", "gdn_commit"]
