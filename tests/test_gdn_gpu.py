"""GatedDeltaNet over tree nodes on the GPU against the float64 oracle
(oracle/gdn.py): gdn_prep, the tree recurrence and the commit replay.

Bars: bf16 outputs (q, k, v, beta, y) within 1e-2 * max|ref| (float32
arithmetic and one bf16 rounding against float64); g within 1e-2 * max|ref|;
the committed state within 1e-4 * max|ref| (float32 state over the path); the
committed conv state bit-exact (a copy)."""

import numpy as np
import pytest
import torch

from gpu_util import assert_close_rel
from oracle import gdn as ogdn

pytestmark = pytest.mark.gpu


def _tree(rng, n, max_depth=8):
    parents, depth = [-1], [0]
    for i in range(1, n):
        while True:
            p = int(rng.integers(0, i))
            if depth[p] < max_depth:
                break
        parents.append(p)
        depth.append(depth[p] + 1)
    return parents


def _f64(t):
    return t.float().cpu().numpy().astype(np.float64)


def _inputs(seed, n, hk, hv):
    g = torch.Generator(device="cuda").manual_seed(seed)
    c = (2 * hk + hv) * 128
    bf = torch.bfloat16
    r = lambda *s, std=1.0: (torch.randn(*s, device="cuda", generator=g) * std).to(bf)  # noqa: E731
    return dict(qkv=r(1, n, c), conv_state=r(1, 3, c), conv_w=r(c, 4, std=0.5), a=r(1, n, hv), b=r(1, n, hv),
                A_log=torch.log(torch.rand(hv, device="cuda", generator=g) * 15 + 1),
                dt_bias=torch.randn(hv, device="cuda", generator=g))


def _deep(n):
    """A 40-node chain with side leaves at depths 21, 35 and 36: walk steps past
    the 32 the tree kernel stages in shared memory, side leaves on both sides."""
    return list(range(-1, 39)) + [34, 35, 20][:n - 40]


@pytest.mark.parametrize("seed,n,hk,hv", [(0, 24, 2, 4), (1, 64, 16, 48), (2, 5, 1, 1), (3, 43, 2, 4)])
def test_prep_recurrence_commit(seed, n, hk, hv):
    from tsb import gdn

    rng = np.random.default_rng(seed)
    parents = _deep(n) if n == 43 else _tree(rng, n)
    x = _inputs(seed, n, hk, hv)
    q, k, v, g, beta = gdn.gdn_prep(x["qkv"], x["conv_state"], gdn.conv_idx(parents, "cuda"), x["conv_w"], x["a"],
                                    x["b"], x["A_log"], x["dt_bias"], hk, 128, hv, 128)
    torch.cuda.synchronize()
    ref = ogdn.prep(_f64(x["qkv"][0]), _f64(x["conv_state"][0]), _f64(x["conv_w"]), _f64(x["a"][0]), _f64(x["b"][0]),
                    _f64(x["A_log"]), _f64(x["dt_bias"]), parents, hk, 128, hv, 128)
    for got, want, name in zip((q[0], k[0], v[0], g[0], beta[0]), ref, ("q", "k", "v", "g", "beta")):
        assert_close_rel(_f64(got), np.asarray(want, np.float64), 1e-2, name)

    # the recurrence, from the GPU's own prep outputs so both sides start from the same values
    gs = torch.Generator(device="cuda").manual_seed(100 + seed)
    state = (torch.randn(1, hv, 128, 128, device="cuda", generator=gs) * 0.1).contiguous()
    y = gdn.tree_gated_delta(q, k, v, g, beta, state, parents)
    torch.cuda.synchronize()
    qf, kf, vf, gf, bf_ = (_f64(t[0]) for t in (q, k, v, g, beta))
    yref = ogdn.tree_recurrence(qf, kf, vf, gf, bf_, _f64(state[0]), parents)
    assert_close_rel(_f64(y[0]), yref, 1e-2, "y")

    # commit the path to the deepest node
    leaf = int(np.argmax([len(ogdn.path(parents, i)) for i in range(n)]))
    nodes = ogdn.path(parents, leaf)
    rec = (x["conv_state"], state, x["qkv"], q, k, v, g, beta)
    conv, st = gdn.gdn_commit(rec, parents, nodes)
    torch.cuda.synchronize()
    sref, cref = ogdn.commit(kf, vf, gf, bf_, _f64(state[0]), x["conv_state"][0].view(torch.int16).cpu().numpy(),
                             x["qkv"][0].view(torch.int16).cpu().numpy(), parents, nodes)
    assert_close_rel(_f64(st[0]), sref, 1e-4, "state")
    assert np.array_equal(conv[0].view(torch.int16).cpu().numpy(), cref)
