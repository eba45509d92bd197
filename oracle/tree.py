"""Tree ancestor masks, restated on the CPU. TEST INFRASTRUCTURE ONLY.

Follows mlx-tree-spec src/mlx_tree_spec/tree_verify.py:66-121 (`Tree`: node 0
is the root with parent -1, every other parent precedes its child; anc[i, j]
is True for j on the root-to-i path, i itself included) and
tree_flash.py:146-148 (`ancestor_bits`: bit j of node i's mask is anc[i, j]).
Extension used by the build: a forest, where any node may have parent -1 (a
root that sees the prefix and itself), as DraftLevel's arbitrary visibility
allows (tree_verify.py:798-806).
"""

from __future__ import annotations

import numpy as np


def check_parents(parents) -> np.ndarray:
    p = np.asarray(parents, dtype=np.int64)
    assert p.ndim == 1 and p.size >= 1
    for i, pi in enumerate(p):
        if not (pi == -1 or 0 <= pi < i):
            raise ValueError(f"parent[{i}] = {pi}: must be -1 or precede the node")
    return p


def ancestors(parents) -> np.ndarray:
    """bool [T, T]: anc[i, j] = j is i or an ancestor of i."""
    p = check_parents(parents)
    t = p.size
    anc = np.zeros((t, t), dtype=bool)
    for i in range(t):
        j = i
        while j != -1:
            anc[i, j] = True
            j = p[j]
    return anc


def ancestor_bits(anc) -> list[int]:
    """Per node the bitmask of tail rows it may see (tree_flash.py:146-148)."""
    return [sum(1 << j for j in range(len(row)) if row[j]) for row in anc]


def ancestor_bits_u64(parents) -> np.ndarray:
    """uint64 [T] bitmasks from a parent array (T <= 64)."""
    anc = ancestors(parents)
    assert anc.shape[0] <= 64
    return np.array(ancestor_bits(anc), dtype=np.uint64)


def depth(parents) -> np.ndarray:
    """int32 [T]: roots 0, children one more than their parent (tree_verify.py:71-75)."""
    p = check_parents(parents)
    d = np.zeros(p.size, dtype=np.int32)
    for i in range(p.size):
        if p[i] >= 0:
            d[i] = d[p[i]] + 1
    return d


def visibility(n_kv: int, tail: int, bits, t: int) -> np.ndarray:
    """bool [T, n_kv]: the reference kernel's rule (tree_flash.py:40-45):
    key gp is visible to query q iff gp < n_kv and (gp < n_kv - tail or bit
    gp - (n_kv - tail) of bits[q] is set). tail == 0: every row visible."""
    vis = np.zeros((t, n_kv), dtype=bool)
    lo = n_kv - tail
    vis[:, :lo] = True
    bits = np.asarray(bits, dtype=np.uint64)
    for q in range(t):
        for j in range(tail):
            if (int(bits[q]) >> j) & 1:
                vis[q, lo + j] = True
    return vis


def additive_mask(parents, offset: int) -> np.ndarray:
    """float32 [T, offset + T]: 0 on the prefix and on ancestors, -inf elsewhere
    (tree_verify.py:131-139)."""
    anc = ancestors(parents)
    t = anc.shape[0]
    m = np.full((t, offset + t), -np.inf, dtype=np.float32)
    m[:, :offset] = 0
    m[:, offset:][anc] = 0
    return m


def mask_bits(mask, tail: int):
    """The inverse of additive_mask / Tree.mask (tree_verify.py:131-139), as
    the build's tsb_tree_mask_bits states it. mask [rows, L]: boolean (True
    visible) or additive float (0 visible, -inf hidden). Returns (bits uint64
    [rows]: bit j set iff column L - tail + j is visible, bad bool [rows]: a
    hidden column before the last `tail`, or an additive value other than 0
    and -inf)."""
    m = np.asarray(mask)
    rows, L = m.shape
    if m.dtype == bool or m.dtype == np.uint8:
        vis = m != 0
        other = np.zeros_like(vis)
    else:
        f = m.astype(np.float64)
        vis = f == 0
        other = ~vis & ~(np.isneginf(f))
    lo = L - tail
    bad = other.any(axis=1) | (~vis[:, :lo]).any(axis=1)
    bits = np.zeros(rows, dtype=np.uint64)
    for r in range(rows):
        bits[r] = np.uint64(sum(1 << j for j in range(tail) if vis[r, lo + j]))
    return bits, bad
