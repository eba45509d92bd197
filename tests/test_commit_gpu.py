"""The tree commit (tsb.keep_kv / tsb_kv_commit) against the CPU oracle
(oracle/kv.take_rows, restating tree_verify.py:487-496 and kv8.py:143-148).

Bar: bit-exact. Every byte of every cache tensor (codes, scales, biases, and
the rows the commit must leave alone) equals the oracle's gather."""

import numpy as np
import pytest
import torch

from oracle import gen, kv

pytestmark = pytest.mark.gpu


def _cache(fmt, b, hkv, cap, seed):
    import tsb

    g = torch.Generator().manual_seed(seed)
    kf = torch.randn(b, hkv, cap, 256, generator=g)
    vf = torch.randn(b, hkv, cap, 256, generator=g)
    from tsb.decoder import make_cache

    c = make_cache(kf.cuda(), vf.cuda(), 0, fmt)
    assert c.kv_format == fmt
    return c


def _tensors(c):
    import tsb

    names = {tsb.TSB_KV_BF16: ("keys", "values"),
             tsb.TSB_KV_REF_Q8_ROW: ("keys", "values", "k_scale", "v_scale"),
             tsb.TSB_KV_MLX_Q8_G64: ("keys", "values", "k_scales", "k_biases", "v_scales", "v_biases")}[c.kv_format]
    return {n: getattr(c, n) for n in names}


def _bytes(t):
    """A tensor's raw bytes as a numpy array of its storage width (bf16 as uint16)."""
    t = t.cpu()
    return t.view(torch.int16).numpy() if t.dtype == torch.bfloat16 else t.numpy()


def _path(parents, node):
    """Root-to-node path of a tree (ascending node indices)."""
    p = []
    while node >= 0:
        p.append(node)
        node = int(parents[node])
    return p[::-1]


@pytest.mark.parametrize("fmt", [0, 1, 2])
def test_keep_kv_per_request(fmt):
    import tsb

    b, hkv, cap = 4, 4, 200
    c = _cache(fmt, b, hkv, cap, seed=fmt)
    before = {n: _bytes(t) for n, t in _tensors(c).items()}
    rng = np.random.default_rng(fmt)
    offs, paths = [], []
    for i in range(b):
        n = [64, 40, 17, 64][i]
        parents = gen.tree_parents(rng, n)
        leaf = int(rng.integers(0, n))
        paths.append(_path(parents, leaf))
        offs.append(int(rng.integers(0, cap - n)))
    paths[0] = list(range(0, 64, 2))[:20]          # far from contiguous, overlapping its destination
    paths[3] = list(range(64))                      # a full-width contiguous path
    new = tsb.keep_kv(c, offs, paths)
    torch.cuda.synchronize()
    assert new == [o + len(p) for o, p in zip(offs, paths)]
    for name, t in _tensors(c).items():
        got, want = _bytes(t), before[name].copy()
        for i in range(b):
            want[i:i + 1] = kv.take_rows(before[name][i:i + 1], offs[i], paths[i])
        assert np.array_equal(got, want), (name, fmt)


@pytest.mark.parametrize("fmt", [0, 1, 2])
def test_keep_kv_reference_form(fmt):
    """One off0 and one path for the whole cache, as the reference calls it;
    a contiguous path moves nothing and only sets the offset."""
    import tsb

    c = _cache(fmt, 2, 4, 96, seed=10 + fmt)
    before = {n: _bytes(t) for n, t in _tensors(c).items()}
    assert tsb.keep_kv(c, 30, [0, 1, 2]) == 33 and c.offset == 33
    torch.cuda.synchronize()
    for name, t in _tensors(c).items():
        assert np.array_equal(_bytes(t), before[name])
    path = [0, 2, 3, 7, 8, 31]
    assert tsb.commit([c], 30, path) == [36] and c.offset == 36
    torch.cuda.synchronize()
    for name, t in _tensors(c).items():
        assert np.array_equal(_bytes(t), kv.take_rows(before[name], 30, path)), (name, fmt)


def test_keep_kv_empty_path_and_declines():
    import tsb

    c = _cache(0, 2, 4, 96, seed=20)
    before = {n: _bytes(t) for n, t in _tensors(c).items()}
    assert tsb.keep_kv(c, [5, 9], [[], [0, 3]]) == [5, 11]
    torch.cuda.synchronize()
    want = before["keys"].copy()
    want[1:2] = kv.take_rows(before["keys"][1:2], 9, [0, 3])
    assert np.array_equal(_bytes(c.keys), want)
    with pytest.raises(tsb.TSBError):
        tsb.keep_kv(c, [0, 0], [[0, 70], [0]])      # node past the 64-node tree width
    with pytest.raises(ValueError):
        tsb.keep_kv(c, [0, 0, 0], [[0], [0], [0]])  # three paths for two requests


def test_commit_many_layers_one_launch():
    """commit() over caches of two formats: one launch per format group, each
    cache equal to the oracle's gather with its own data."""
    import tsb

    caches = [_cache(fmt, 3, 2, 80, seed=30 + i) for i, fmt in enumerate((1, 1, 0, 1, 0))]
    before = [{n: _bytes(t) for n, t in _tensors(c).items()} for c in caches]
    offs = [5, 11, 40]
    paths = [[0, 3, 4, 9], [0, 1, 2, 3, 7], [0, 2]]
    out = tsb.commit(caches, offs, paths)
    torch.cuda.synchronize()
    assert out == [[9, 16, 42]] * len(caches)
    for c, b0 in zip(caches, before):
        for name, t in _tensors(c).items():
            want = b0[name].copy()
            for i in range(3):
                want[i:i + 1] = kv.take_rows(b0[name][i:i + 1], offs[i], paths[i])
            assert np.array_equal(_bytes(t), want), name
