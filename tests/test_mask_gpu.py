"""SDPA masks on the GPU: tsb_tree_mask_bits against the oracle's inverse of
Tree.mask (mlx-tree-spec src/mlx_tree_spec/tree_verify.py:131-139), and the
mlx-lm SDPA hook (long_attention.py:69-88) against tree_flash with parents."""

import numpy as np
import pytest
import torch

from gpu_util import dev
from oracle import gen, tree

pytestmark = pytest.mark.gpu

_TORCH = {"bool": torch.bool, "bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def _to_dev(m: np.ndarray, dtype: str) -> torch.Tensor:
    if dtype == "bool":
        return dev(m == 0)
    return dev(m.astype(np.float32)).to(_TORCH[dtype])


@pytest.mark.parametrize("dtype", ["bool", "bf16", "f16", "f32"])
@pytest.mark.parametrize("t,off", [(1, 0), (7, 1000), (33, 5003), (64, 40)])
def test_mask_bits_matches_oracle(dtype, t, off):
    import tsb

    rng = np.random.default_rng(t * 7919 + off)
    p = gen.tree_parents(rng, t)
    m = tree.additive_mask(p, off)
    if t > 2 and dtype != "bool":
        m[1, off] = -1.0  # a bias on a tree column
        m[2, 0] = -np.inf if off else m[2, 0]  # a hidden prefix column
    if t > 5 and dtype != "bool":
        m[4, off + 2] = np.inf
        m[5, off // 2] = np.nan
    want_bits, want_bad = tree.mask_bits(m, t)
    bits, bad = tsb.mask_bits(_to_dev(m, dtype), t)
    torch.cuda.synchronize()
    got = bits.cpu().numpy().view(np.uint64)
    ok = ~want_bad
    assert np.array_equal(got[ok], want_bits[ok])
    assert int(bad.item()) == int(want_bad.sum())


def test_mask_bits_batched_and_strided():
    import tsb

    rng = np.random.default_rng(5)
    t, off = 32, 777
    ms = np.stack([tree.additive_mask(gen.tree_parents(rng, t), off) for _ in range(4)])
    wide = torch.full((4, t, off + t + 13), float("-inf"), device="cuda", dtype=torch.bfloat16)
    wide[..., :off + t] = dev(ms).to(torch.bfloat16)
    view = wide[..., :off + t]  # rows off + t + 13 elements apart
    bits, bad = tsb.mask_bits(view, t)
    torch.cuda.synchronize()
    assert bits.shape == (4, t) and int(bad.item()) == 0
    got = bits.cpu().numpy().view(np.uint64)
    for b in range(4):
        assert np.array_equal(got[b], tree.mask_bits(ms[b], t)[0])
    # a tail longer than 64 rows is declined
    assert tsb.mask_bits(view, 65) is None


def _bf16_cache(bsz, hkv, L, d, seed):
    import tsb

    g = torch.Generator(device="cuda").manual_seed(seed)
    k = torch.randn(bsz, hkv, L, d, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(bsz, hkv, L, d, device="cuda", generator=g).to(torch.bfloat16)
    return tsb.KVCache(k, v, L), k, v


@pytest.mark.parametrize("dtype", ["bf16", "bool"])
def test_sdpa_hook_tree_mask_equals_parents(dtype):
    """Tree.mask handed to the hook gives the same bits as the parent array,
    so the output is the same launch's bit for bit."""
    import tsb

    t, off, hq, hkv, d = 32, 3000, 24, 4, 256
    cache, k, v = _bf16_cache(1, hkv, off + t, d, seed=21)
    q = torch.randn(1, hq, t, d, device="cuda", generator=torch.Generator(device="cuda").manual_seed(22))
    q = q.to(torch.bfloat16)
    p = gen.tree_parents(np.random.default_rng(23), t)
    want = tsb.tree_flash(q, cache, d**-0.5, parents=dev(p.astype(np.int32)))
    got = tsb.sdpa(q, k, v, cache, d**-0.5, _to_dev(tree.additive_mask(p, off), dtype))
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    # the same mask as (B, 1, n, L), mlx-lm's broadcast layout
    got4 = tsb.sdpa(q, k, v, cache, d**-0.5, _to_dev(tree.additive_mask(p, off), dtype)[None, None])
    torch.cuda.synchronize()
    assert torch.equal(got4, want)


@pytest.mark.parametrize("fmt", ["bf16", "mlx_q8"])
def test_sdpa_hook_causal_equals_chain(fmt):
    import tsb

    t, off, hq, hkv, d = 8, 2000, 24, 4, 256
    cache, k, v = _bf16_cache(2, hkv, off + t, d, seed=31)
    if fmt == "mlx_q8":
        kw, ks, kb = tsb.quantize_g64(k.float())
        vw, vs, vb = tsb.quantize_g64(v.float())
        cache = tsb.MLXQ8KVCache(kw, vw, ks, kb, vs, vb, off + t)
    q = torch.randn(2, hq, t, d, device="cuda", generator=torch.Generator(device="cuda").manual_seed(32))
    q = q.to(torch.bfloat16)
    chain = dev(gen.chain_parents(t).astype(np.int32))
    want = tsb.tree_flash(q, cache, d**-0.5, parents=chain)
    for mask in (None, "causal"):
        got = tsb.sdpa(q, k, v, cache, d**-0.5, mask)
        torch.cuda.synchronize()
        assert torch.equal(got, want), mask


def test_sdpa_hook_without_cache_is_causal_attention():
    """cache None: keys/values are all the keys (a prefill chunk of n <= 64)."""
    import tsb

    t, hq, hkv, d = 16, 24, 4, 256
    _, k, v = _bf16_cache(1, hkv, t, d, seed=41)
    q = torch.randn(1, hq, t, d, device="cuda", generator=torch.Generator(device="cuda").manual_seed(42))
    q = q.to(torch.bfloat16)
    got = tsb.sdpa(q, k, v, None, d**-0.5, "causal")
    g = hq // hkv
    ref = torch.nn.functional.scaled_dot_product_attention(
        q.float(), k.float().repeat_interleave(g, 1), v.float().repeat_interleave(g, 1), is_causal=True,
        scale=d**-0.5)
    torch.cuda.synchronize()
    err = (got.float() - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item()


def test_sdpa_hook_declines_to_fallback():
    import tsb

    t, off, hq, hkv, d = 4, 100, 24, 4, 256
    cache, k, v = _bf16_cache(1, hkv, off + t, d, seed=51)
    q = torch.zeros(1, hq, t, d, device="cuda", dtype=torch.bfloat16)
    calls = []

    def fallback(queries, keys, values, *args, cache=None, scale=None, mask=None, **kwargs):
        calls.append((mask, args, kwargs))
        return "fallback"

    m = tree.additive_mask(gen.chain_parents(t), off)
    m[0, 3] = -2.5  # a real additive bias: not a visibility mask
    biased = _to_dev(m, "bf16")
    assert tsb.sdpa(q, k, v, cache, 0.1, biased, fallback=fallback) == "fallback"
    assert tsb.sdpa(q, k, v, cache, 0.1, biased) is None
    per_head = _to_dev(tree.additive_mask(gen.chain_parents(t), off), "bf16")[None, None].expand(1, hq, t, off + t)
    assert tsb.sdpa(q, k, v, cache, 0.1, per_head, fallback=fallback) == "fallback"
    assert tsb.sdpa(q, k, v, cache, 0.1, "sliding", fallback=fallback) == "fallback"
    assert tsb.sdpa(q, k, v, cache, 0.1, None, 7, fallback=fallback) == "fallback"
    assert len(calls) == 4 and calls[-1][1] == (7,)
