"""GPU parity of tree masks and tree-mask attention against the oracle.

Bar: ancestor masks bit-exact; attention max-abs-err <= 2e-2 * max|ref| for
the bf16 output, and lse within 1e-2 absolute."""

import glob
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, load_golden
from gpu_util import assert_close_rel, dev, dev_bf16, dev_u32, host_f32
from oracle import attention, bf16, gen, kv, tree

pytestmark = pytest.mark.gpu


def test_ancestor_bits_bit_exact():
    import tsb

    g = load_golden("ancestors.npz")
    for key in [k[: -len("_parents")] for k in g if k.endswith("_parents")]:
        bits, depth = tsb.ancestor_bits(dev(g[f"{key}_parents"]), depth=True)
        torch.cuda.synchronize()
        assert np.array_equal(bits.cpu().numpy().view(np.uint64), g[f"{key}_bits"]), key
        assert np.array_equal(depth.cpu().numpy(), g[f"{key}_depth"]), key


def test_ancestor_bits_batched_and_invalid():
    import tsb

    p = np.stack([gen.tree_parents(np.random.default_rng(i), 40) for i in range(4)])
    bad = p[1].copy()
    bad[7] = 9  # not an earlier node
    p[1] = bad
    bits, depth = tsb.ancestor_bits(dev(p), depth=True)
    torch.cuda.synchronize()
    bits = bits.cpu().numpy().view(np.uint64)
    for i in (0, 2, 3):
        assert np.array_equal(bits[i], tree.ancestor_bits_u64(p[i]))
    assert bits[1, 7] == 0 and depth.cpu().numpy()[1, 7] == -1


def _cache_from_fixture(g):
    import tsb

    fmt = str(g["fmt"])
    n_kv = int(g["n_kv"])
    if fmt == "bf16":
        return tsb.KVCache(dev_bf16(g["k"]), dev_bf16(g["v"]), n_kv)
    if fmt == "ref_q8":
        return tsb.Q8KVCache(dev(g["k"]), dev(g["v"]), dev(g["k_scale"]), dev(g["v_scale"]), n_kv)
    return tsb.MLXQ8KVCache(dev_u32(g["k"]), dev_u32(g["v"]), dev_bf16(g["k_scales"]), dev_bf16(g["k_biases"]),
                            dev_bf16(g["v_scales"]), dev_bf16(g["v_biases"]), n_kv)


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "attn_*.npz"))), ids=os.path.basename)
@pytest.mark.parametrize("mask_from", ["parents", "bits"])
def test_attn_golden(path, mask_from):
    import tsb

    g = load_golden(os.path.basename(path))
    cache = _cache_from_fixture(g)
    q = dev_bf16(g["q"])
    t = q.shape[2]
    tail = int(g["tail"])
    if mask_from == "parents":
        if tail != t:
            pytest.skip("explicit-mask fixture (tail longer than the query count)")
        res = tsb.tree_flash(q, cache, float(g["scale"]), parents=dev(g["parents"]), stats=True)
    else:
        bits = torch.from_numpy(g["bits"].view(np.int64)).cuda()
        res = tsb.tree_flash(q, cache, float(g["scale"]), bits, tail=tail, stats=True)
    assert res is not None
    out, maxs, sums = res
    torch.cuda.synchronize()
    assert_close_rel(host_f32(out), g["out"], 2e-2, path)
    assert np.allclose(host_f32(maxs)[..., 0], g["lse"], atol=1e-2)
    assert np.all(host_f32(sums) == 1.0)


def _full_case(bsz, L, fmt, seed, t=32, hq=24, hkv=4, d=256, heads_checked=(0, 13, 23)):
    """The attention benchmark shape (T=32, 24q/4kv heads, D=256) at full size; the
    oracle checks a few query heads."""
    import tsb

    torch.manual_seed(seed)
    n_kv = L + t
    cap = n_kv + 32
    kf = torch.randn(bsz, hkv, cap, d, device="cuda")
    vf = torch.randn(bsz, hkv, cap, d, device="cuda")
    q = torch.randn(bsz, hq, t, d, device="cuda").to(torch.bfloat16)
    if fmt == "bf16":
        kb, vb = kf.to(torch.bfloat16), vf.to(torch.bfloat16)
        cache = tsb.KVCache(kb, vb, n_kv)
        kval, vval = kb.float(), vb.float()
    elif fmt == "ref_q8":
        kq, ksc = tsb.quantize_rows(kf)
        vq, vsc = tsb.quantize_rows(vf)
        cache = tsb.Q8KVCache(kq, vq, ksc, vsc, n_kv)
        kval = torch.from_numpy(kv.dequant_rows(kq.cpu().numpy(), ksc.cpu().numpy())).float()
        vval = torch.from_numpy(kv.dequant_rows(vq.cpu().numpy(), vsc.cpu().numpy())).float()
    else:
        kw, ks, kbias = tsb.quantize_g64(kf)
        vw, vs, vbias = tsb.quantize_g64(vf)
        cache = tsb.MLXQ8KVCache(kw, vw, ks, kbias, vs, vbias, n_kv)
        kval = torch.from_numpy(kv.dequant_g64(kw.cpu().numpy().view(np.uint32), bf16.from_torch_bf16(ks),
                                               bf16.from_torch_bf16(kbias))).float()
        vval = torch.from_numpy(kv.dequant_g64(vw.cpu().numpy().view(np.uint32), bf16.from_torch_bf16(vs),
                                               bf16.from_torch_bf16(vbias))).float()
    rng = np.random.default_rng(seed)
    parents = np.stack([gen.tree_parents(rng, t) for _ in range(bsz)])
    out = tsb.tree_flash(q, cache, d**-0.5, parents=dev(parents))
    torch.cuda.synchronize()
    got = host_f32(out)
    bits = np.stack([tree.ancestor_bits_u64(p) for p in parents])
    qn = host_f32(q)
    kvn, vvn = kval.cpu().numpy(), vval.cpu().numpy()
    g = hq // hkv
    for h in heads_checked:
        ref = attention.tree_attention(qn[:, h:h + 1], kvn[:, h // g:h // g + 1], vvn[:, h // g:h // g + 1], n_kv, t,
                                       bits, d**-0.5)
        assert_close_rel(got[:, h:h + 1], ref, 2e-2, f"L={L} fmt={fmt} head {h}")


@pytest.mark.parametrize("bsz,L", [(1, 1024), (4, 1024), (1, 8192), (4, 8192), (1, 32768)])
def test_attn_config4_bf16(bsz, L):
    _full_case(bsz, L, "bf16", seed=100 + bsz + L)


@pytest.mark.parametrize("bsz,L", [(1, 1024), (4, 8192), (1, 32768)])
def test_attn_config4_mlx_q8(bsz, L):
    _full_case(bsz, L, "mlx_q8", seed=200 + bsz + L)


@pytest.mark.parametrize("bsz,L", [(1, 1024), (4, 8192), (1, 32768)])
def test_attn_config4_ref_q8(bsz, L):
    _full_case(bsz, L, "ref_q8", seed=300 + bsz + L)


def _cache_with_tail_rows(fmt, n_kv, cap, fill, seed, bsz=2, hkv=4, d=256):
    """A cache whose rows >= n_kv hold `fill` (bf16 values, or the 8-bit
    formats' scales); rows < n_kv are the same for every fill."""
    import tsb

    g = torch.Generator(device="cuda").manual_seed(seed)
    kf = torch.randn(bsz, hkv, cap, d, device="cuda", generator=g)
    vf = torch.randn(bsz, hkv, cap, d, device="cuda", generator=g)
    if fmt == "bf16":
        kb, vb = kf.to(torch.bfloat16), vf.to(torch.bfloat16)
        kb[:, :, n_kv:] = fill
        vb[:, :, n_kv:] = fill
        return tsb.KVCache(kb, vb, n_kv)
    if fmt == "ref_q8":
        kq, ksc = tsb.quantize_rows(kf)
        vq, vsc = tsb.quantize_rows(vf)
        ksc[:, :, n_kv:] = fill
        vsc[:, :, n_kv:] = fill
        return tsb.Q8KVCache(kq, vq, ksc, vsc, n_kv)
    kw, ks, kbias = tsb.quantize_g64(kf)
    vw, vs, vbias = tsb.quantize_g64(vf)
    for t in (ks, kbias, vs, vbias):
        t[:, :, n_kv:] = fill
    return tsb.MLXQ8KVCache(kw, vw, ks, kbias, vs, vbias, n_kv)


@pytest.mark.parametrize("fmt", ["bf16", "ref_q8", "mlx_q8"])
@pytest.mark.parametrize("n_kv", [1000, 1024 + 7])
def test_attn_rows_past_n_kv_never_read_into_output(fmt, n_kv):
    """Cache rows at or past n_kv (here NaN, inside the same tile as the last
    keys) leave the output bit-identical to a cache with zeros there."""
    import tsb

    cap = n_kv + 40
    t, hq = 16, 24
    q = torch.randn(2, hq, t, 256, device="cuda").to(torch.bfloat16)
    rng = np.random.default_rng(n_kv)
    parents = dev(np.stack([gen.tree_parents(rng, t) for _ in range(2)]))
    outs = []
    for fill in (0.0, float("nan")):
        cache = _cache_with_tail_rows(fmt, n_kv, cap, fill, seed=n_kv)
        outs.append(tsb.tree_flash(q, cache, 256**-0.5, parents=parents))
    torch.cuda.synchronize()
    assert not torch.isnan(outs[1].float()).any()
    assert torch.equal(outs[0], outs[1])


def test_attn_mlx_q8_odd_capacity():
    """MLX 8-bit caches with an odd capacity take the warp-MMA kernel; the
    results meet the same bar."""
    import tsb

    torch.manual_seed(7)
    t, hq, hkv, d, n_kv = 8, 24, 4, 256, 700
    cap = 701
    kf = torch.randn(1, hkv, cap, d, device="cuda")
    vf = torch.randn(1, hkv, cap, d, device="cuda")
    q = torch.randn(1, hq, t, d, device="cuda").to(torch.bfloat16)
    kw, ks, kbias = tsb.quantize_g64(kf)
    vw, vs, vbias = tsb.quantize_g64(vf)
    cache = tsb.MLXQ8KVCache(kw, vw, ks, kbias, vs, vbias, n_kv)
    rng = np.random.default_rng(7)
    parents = gen.tree_parents(rng, t)[None]
    out = tsb.tree_flash(q, cache, d**-0.5, parents=dev(parents))
    torch.cuda.synchronize()
    kval = kv.dequant_g64(kw.cpu().numpy().view(np.uint32), bf16.from_torch_bf16(ks), bf16.from_torch_bf16(kbias))
    vval = kv.dequant_g64(vw.cpu().numpy().view(np.uint32), bf16.from_torch_bf16(vs), bf16.from_torch_bf16(vbias))
    bits = tree.ancestor_bits_u64(parents[0])[None]
    ref = attention.tree_attention(host_f32(q), kval, vval, n_kv, t, bits, d**-0.5)
    assert_close_rel(host_f32(out), ref, 2e-2, "odd capacity")


def test_attn_declines():
    import tsb

    q = torch.zeros(1, 4, 2, 128, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(1, 1, 16, 128, dtype=torch.bfloat16, device="cuda")
    assert tsb.tree_flash(q, tsb.KVCache(k, k, 8), 0.1, parents=torch.tensor([-1, 0], device="cuda")) is None
