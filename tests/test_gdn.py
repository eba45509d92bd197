"""GatedDeltaNet walks and the C ABI's host-side checks, on the CPU.

The walk layout (tsb.gdn.walks) must cover every node, give each node one
owner that really holds it, fold a side leaf only onto a walk through its
parent at the step before, and build the causal-conv windows exactly as the
oracle does (oracle/gdn.conv_window, restating tree_verify.py:111-118)."""

import ctypes

import numpy as np
import pytest

from oracle import gdn as ogdn


def _tree(rng, n, max_depth=8):
    parents = [-1]
    depth = [0]
    for i in range(1, n):
        while True:
            p = int(rng.integers(0, i))
            if depth[p] < max_depth:
                break
        parents.append(p)
        depth.append(depth[p] + 1)
    return parents


@pytest.mark.parametrize("seed,n", [(0, 1), (1, 8), (2, 32), (3, 64), (4, 64)])
def test_walks_cover_every_node(seed, n):
    from tsb.gdn import walks

    rng = np.random.default_rng(seed)
    parents = _tree(rng, n)
    w = walks(parents)
    held = [set() for _ in range(n)]
    for r, (rp, rs) in enumerate(zip(w.rows, w.sibs)):
        assert rp == tuple(ogdn.path(parents, rp[-1]))       # a walk is a root path
        assert len(rs) == len(rp)
        for t, s in enumerate(rs):
            if s >= 0:
                assert t >= 1 and parents[s] == rp[t - 1]     # a side leaf hangs off the walk's previous node
                held[s].add(r)
        for i in rp:
            held[i].add(r)
    for i in range(n):
        assert held[i], f"node {i} in no walk"
        assert w.owner[i] in held[i]
    assert w.lmax == max(len(r) for r in w.rows)
    assert len(w.rows) <= sum(1 for i in range(n) if i not in set(parents))
    assert np.array_equal(w.conv_idx, ogdn.conv_window(parents))


def test_walks_chain_and_star():
    from tsb.gdn import walks

    chain = walks([-1, 0, 1, 2, 3])
    assert chain.rows == ((0, 1, 2, 3, 4),) and chain.lmax == 5
    assert all(s == -1 for s in chain.sibs[0])
    star = walks([-1, 0, 0, 0, 1])      # leaves 2, 3 hang off the root, 4 under 1
    assert len(star.rows) == 2           # 3 rides on walk 0-2 as its side leaf; 4 needs its own walk
    with pytest.raises(ValueError):
        walks([0, 0])
    with pytest.raises(ValueError):
        walks([-1, 1])


def test_conv_window_reaches_into_the_conv_state():
    w = ogdn.conv_window([-1, 0, 1])
    assert w.tolist() == [[0, 1, 2, 3], [1, 2, 3, 4], [2, 3, 4, 5]]


def test_abi_host_checks():
    import tsb

    lib = tsb._lib.load()
    E = tsb._lib
    f = 0x1000
    nodes = (ctypes.c_int32 * 2)(0, 1)
    # prep: heads of 64 decline; Hv not a multiple of Hk declines; a missing pointer is a contract violation
    assert lib.tsb_gdn_prep(f, f, f, f, f, f, f, f, f, f, f, f, f, 4, 2, 64, 4, 64, None) == E.TSB_EUNSUPPORTED
    assert lib.tsb_gdn_prep(f, f, f, f, f, f, f, f, f, f, f, f, f, 4, 3, 128, 4, 128, None) == E.TSB_EUNSUPPORTED
    assert lib.tsb_gdn_prep(None, f, f, f, f, f, f, f, f, f, f, f, f, 4, 2, 128, 4, 128, None) == E.TSB_EINVAL
    assert lib.tsb_gdn_prep(f, f, f, f, f, f, f, f, f, f, f, f, f, 0, 2, 128, 4, 128, None) == E.TSB_EINVAL
    # tree: empty walk arrays, misaligned state
    assert lib.tsb_tree_gated_delta(f, f, f, f, f, f, f, f, f, 0, 4, 8, 2, 128, 4, 128, f, None) == E.TSB_EINVAL
    assert lib.tsb_tree_gated_delta(f, f, f, f, f, f + 8, f, f, f, 2, 4, 8, 2, 128, 4, 128, f, None) == E.TSB_EINVAL
    assert lib.tsb_tree_gated_delta(f, f, f, f, f, f, f, f, f, 2, 4, 8, 2, 128, 4, 96, f, None) == E.TSB_EUNSUPPORTED
    # prep: more nodes than one grid dimension holds
    assert lib.tsb_gdn_prep(f, f, f, f, f, f, f, f, f, f, f, f, f, 65536, 2, 128, 4, 128, None) == E.TSB_EUNSUPPORTED
    # commit: a path node outside the tree, an empty path, a path longer than 64
    o = 0x1000000  # conv_out apart from conv_state
    assert lib.tsb_gdn_commit(f, f, f, f, f, f, f, f, nodes, 2, 1, 2, 128, 4, 128, f, o, None) == E.TSB_EINVAL
    assert lib.tsb_gdn_commit(f, f, f, f, f, f, f, f, nodes, 0, 8, 2, 128, 4, 128, f, o, None) == E.TSB_EINVAL
    long = (ctypes.c_int32 * 65)(*range(65))
    assert lib.tsb_gdn_commit(f, f, f, f, f, f, f, f, long, 65, 80, 2, 128, 4, 128, f, o, None) == E.TSB_EUNSUPPORTED
    # commit: conv_out overlapping conv_state ([3, (2*2 + 4) * 128] bf16 = 6144 bytes)
    cs = 0x100000
    for out in (cs, cs + 6142, cs - 6142):
        assert lib.tsb_gdn_commit(f, f, f, f, f, cs, f, f, nodes, 2, 8, 2, 128, 4, 128, f, out, None) == E.TSB_EINVAL


def test_walks_take_a_tree_object():
    from tsb.gdn import walks

    class Tree:
        parents = (-1, 0, 0, 1)

    a, b = walks(Tree()), walks([-1, 0, 0, 1])
    assert (a.rows, a.sibs, a.owner, a.lmax) == (b.rows, b.sibs, b.owner, b.lmax)
    assert np.array_equal(a.conv_idx, b.conv_idx)
