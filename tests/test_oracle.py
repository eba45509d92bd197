"""The CPU oracle, pinned against the reference's own known answers and code,
and checked for internal consistency. No GPU."""

import glob
import os

import numpy as np
import pytest

from conftest import GOLDEN, load_golden
from oracle import attention, bf16, gen, kv, qmm, tree


# ---------------------------------------------------------------- bf16 helpers

def test_bf16_round_trip_and_rne():
    vals = np.array([0.0, -0.0, 1.0, 1.00390625, 1.01171875, 3.14159, -2.5e-3, 65504.0, 1e30], dtype=np.float32)
    bits = bf16.f32_to_bf16_bits(vals)
    back = bf16.bf16_bits_to_f32(bits)
    assert np.all(np.abs(back - vals) <= np.abs(vals) * 2.0**-8)
    # ties to even: 1 + 2^-8 is halfway between 1 and 1 + 2^-7 -> 1 (even mantissa)
    assert bf16.bf16_bits_to_f32(bf16.f32_to_bf16_bits(np.float32(1 + 2**-8)))[()] == 1.0
    # 1 + 3*2^-8 is halfway between 1+2^-7 and 1+2^-6 -> 1+2^-6 (even)
    assert bf16.bf16_bits_to_f32(bf16.f32_to_bf16_bits(np.float32(1 + 3 * 2**-8)))[()] == np.float32(1 + 2**-6)


def test_bf16_matches_torch():
    import torch

    x = np.random.default_rng(0).standard_normal(10000).astype(np.float32) * 100
    ours = bf16.f32_to_bf16_bits(x)
    theirs = bf16.from_torch_bf16(torch.from_numpy(x).to(torch.bfloat16))
    assert np.array_equal(ours, theirs)


# ---------------------------------------------------------------- weight format

def test_pack_unpack_round_trip():
    rng = np.random.default_rng(1)
    for bits in (4, 8):
        q = rng.integers(0, 1 << bits, size=(7, 64), dtype=np.uint8)
        w = qmm.pack_bits(q, bits)
        assert w.shape == (7, 64 * bits // 32) and w.dtype == np.uint32
        assert np.array_equal(qmm.unpack_bits(w, bits), q)


def test_nibble_order_matches_reference_kernels():
    """Element i of a word is `(word >> (4*i)) & 0xF` (qmm_packed.py:200-201,
    348-349, 635-636): element 8c + i of the row."""
    q = np.arange(16, dtype=np.uint8)[None, :] % 16
    w = qmm.pack_bits(q, 4)
    for c in range(2):
        for i in range(8):
            assert (int(w[0, c]) >> (4 * i)) & 0xF == q[0, 8 * c + i]


def test_pack_nax_relayout_is_a_permutation():
    """The reference's load-time relayout (qmm_packed.py:223-232) and its
    inverse (packed_linear.py:72-80) restated on numpy arrays: a pure
    permutation of the MLX words, so consuming MLX's layout directly loses
    nothing."""
    rng = np.random.default_rng(2)
    n, kw = 64, 32
    w = rng.integers(0, 2**32, size=(n, kw), dtype=np.uint64).astype(np.uint32)
    wq2 = w.reshape(n // 32, 32, kw // 2, 2).transpose(0, 2, 1, 3).reshape(-1)
    back = wq2.reshape(n // 32, kw // 2, 32, 2).transpose(0, 2, 1, 3).reshape(n, kw)
    assert np.array_equal(back, w)


def test_quantize_dequantize_error_bound():
    rng = np.random.default_rng(3)
    w = rng.standard_normal((32, 256)).astype(np.float32) * 0.02
    wq, s, b = qmm.quantize(w)
    deq = bf16.bf16_bits_to_f32(qmm.dequantize(wq, s, b))
    step = np.repeat(bf16.bf16_bits_to_f32(s), 64, axis=-1)
    assert np.all(np.abs(deq - w) <= 0.5 * step + np.abs(w) * 2**-7 + 1e-6)


def test_dequant_rule_is_fp32_fma_then_bf16():
    """bf16_rne(fmaf(q, s, b)) for q in 0..15 and adversarial s, b."""
    import math

    rng = np.random.default_rng(4)
    s_bits = bf16.f32_to_bf16_bits(rng.standard_normal(200).astype(np.float32) * 0.01)
    b_bits = bf16.f32_to_bf16_bits(rng.standard_normal(200).astype(np.float32) * 0.1)
    # include extreme exponent spreads where float64 q*s+b is inexact
    s_bits[:4] = bf16.f32_to_bf16_bits(np.array([1e-30, 3e-20, 1e20, 7e-5], dtype=np.float32))
    b_bits[:4] = bf16.f32_to_bf16_bits(np.array([1.0, -3.0, 1e-20, 1e10], dtype=np.float32))
    q = rng.integers(0, 16, size=(200, 64), dtype=np.uint8)
    w = qmm.pack_bits(q, 4)
    deq = qmm.dequantize(w, s_bits[:, None], b_bits[:, None])
    sf, bf = bf16.bf16_bits_to_f32(s_bits), bf16.bf16_bits_to_f32(b_bits)
    for r in range(0, 200, 7):
        for kk in range(0, 64, 5):
            if hasattr(math, "fma"):
                f = np.float32(math.fma(float(q[r, kk]), float(sf[r]), float(bf[r])))
            else:  # exact rational arithmetic, then one rounding to float32
                from fractions import Fraction

                exact = Fraction(int(q[r, kk])) * Fraction(float(sf[r])) + Fraction(float(bf[r]))
                f = np.float32(float(exact))  # float() of a Fraction rounds correctly to double;
                # double -> float32 can double-round only when the double is inexact; guard that case
                if Fraction(float(exact)) != exact:
                    continue
            assert deq[r, kk] == bf16.f32_to_bf16_bits(f)[()]


def test_qmv_decomposition_identity():
    """The reference's GEMV identity sum_k (s q + b) x = s sum q x + b sum x
    (qmm_packed.py:14-16, 424-425) holds for the oracle's exact qmm."""
    rng = np.random.default_rng(5)
    x = gen.x_bf16(rng, 3, 256)
    wq, s, b = gen.weights_w4g64(rng, 128, 256)
    y = qmm.qmm(x, wq, s, b)
    xf = bf16.bf16_bits_to_f32(x).astype(np.float64).reshape(3, 4, 64)
    q = qmm.unpack_bits(wq, 4).astype(np.float64).reshape(128, 4, 64)
    sf = bf16.bf16_bits_to_f32(s).astype(np.float64)
    bf = bf16.bf16_bits_to_f32(b).astype(np.float64)
    y2 = np.einsum("ng,mng->mn", sf, np.einsum("ngk,mgk->mng", q, xf)) + np.einsum("ng,mg->mn", bf, xf.sum(-1))
    # the oracle rounds each dequantized weight to bf16; the identity is exact arithmetic
    assert np.max(np.abs(y - y2)) <= 2e-2 * np.max(np.abs(y))


# ---------------------------------------------------------------- tree masks

def test_ancestor_bits_reference_known_answer():
    """tests/test_units.py:29-32 of the reference: root 0, children 1 and 2 of 0."""
    anc = [[1, 0, 0], [1, 1, 0], [1, 0, 1]]
    assert tree.ancestor_bits(anc) == [0b001, 0b011, 0b101]
    assert list(tree.ancestor_bits_u64([-1, 0, 0])) == [0b001, 0b011, 0b101]


def test_tree_matches_reference_walk():
    """anc[i, path(i)] = True with path() walking parents to the root
    (tree_verify.py:84-112); depth[i] = depth[parent] + 1 (71-75)."""
    p = gen.tree_parents(np.random.default_rng(6), 32)
    anc = tree.ancestors(p)
    d = tree.depth(p)
    for i in range(32):
        path = []
        j = i
        while j != -1:
            path.append(j)
            j = p[j]
        assert set(np.nonzero(anc[i])[0]) == set(path)
        assert d[i] == len(path) - 1 and d[i] <= 8


def test_chain_and_forest_masks():
    bits = tree.ancestor_bits_u64(gen.chain_parents(5))
    assert list(bits) == [(1 << (q + 1)) - 1 for q in range(5)]  # kv8.causal_bits (kv8.py:194-197)
    bits = tree.ancestor_bits_u64([-1, 0, -1, 2])
    assert list(bits) == [0b0001, 0b0011, 0b0100, 0b1100]
    with pytest.raises(ValueError):
        tree.ancestors([-1, 2, 0])


def test_visibility_equals_additive_mask():
    """The bitmask rule (tree_flash.py:40-45) equals Tree.mask's additive mask
    (tree_verify.py:131-139) when the tail is the nodes themselves."""
    p = gen.tree_parents(np.random.default_rng(7), 12)
    off = 20
    vis = tree.visibility(off + 12, 12, tree.ancestor_bits_u64(p), 12)
    assert np.array_equal(vis, tree.additive_mask(p, off) == 0)



def test_mask_bits_inverts_additive_mask():
    """Tree.mask (tree_verify.py:131-139) read back as bits gives the tree's
    ancestor bits; the boolean form the same; a bias value or a hidden prefix
    column is flagged."""
    rng = np.random.default_rng(11)
    for t, off in [(1, 0), (5, 3), (17, 40), (64, 9)]:
        p = gen.tree_parents(rng, t)
        m = tree.additive_mask(p, off)
        bits, bad = tree.mask_bits(m, t)
        assert np.array_equal(bits, tree.ancestor_bits_u64(p)) and not bad.any()
        bits_b, bad_b = tree.mask_bits(m == 0, t)
        assert np.array_equal(bits_b, bits) and not bad_b.any()
    m = tree.additive_mask([-1, 0, 1], 4)
    m[1, 5] = -1.0  # a bias inside the tree rows
    m[2, 0] = -np.inf  # a hidden prefix column
    bits, bad = tree.mask_bits(m, 3)
    assert list(bad) == [False, True, True]
    assert int(bits[0]) == 1

def test_golden_ancestors_regenerate():
    g = load_golden("ancestors.npz")
    for key in [k[: -len("_parents")] for k in g if k.endswith("_parents")]:
        p = g[f"{key}_parents"]
        assert np.array_equal(tree.ancestor_bits_u64(p), g[f"{key}_bits"])
        assert np.array_equal(tree.depth(p), g[f"{key}_depth"])
    assert list(g["reference_known_answer_bits"]) == [1, 3, 5]


# ---------------------------------------------------------------- attention

def _sdpa_additive(q, k, v, mask, scale):
    s = np.einsum("td,jd->tj", q, k) * scale + mask
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s)
    return (p / p.sum(-1, keepdims=True)) @ v


def test_tree_attention_equals_masked_sdpa():
    """tree_flash vs MLX SDPA with the additive tree mask is the reference's own
    cross-check (bench/attn/flash_bench.py:58-64)."""
    rng = np.random.default_rng(8)
    t, L, d, hq, hkv = 6, 40, 16, 4, 2
    p = gen.tree_parents(rng, t)
    q = rng.standard_normal((1, hq, t, d))
    k = rng.standard_normal((1, hkv, L + t, d))
    v = rng.standard_normal((1, hkv, L + t, d))
    out = attention.tree_attention(q, k, v, L + t, t, tree.ancestor_bits_u64(p), d**-0.5)
    mask = tree.additive_mask(p, L)
    for h in range(hq):
        ref = _sdpa_additive(q[0, h], k[0, h // 2], v[0, h // 2], mask, d**-0.5)
        assert np.allclose(out[0, h], ref, atol=1e-12)


def test_block_merge_identity():
    """Per-block (max, sum) statistics rebuild the full softmax
    (tree_verify.py:389-401)."""
    rng = np.random.default_rng(9)
    s = rng.standard_normal((3, 50)) * 3
    v = rng.standard_normal((50, 8))
    full = (np.exp(s - s.max(-1, keepdims=True)) / np.exp(s - s.max(-1, keepdims=True)).sum(-1, keepdims=True)) @ v
    blocks = [(0, 17), (17, 30), (30, 50)]
    outs, maxs, sums = [], [], []
    for a, b in blocks:
        m = s[:, a:b].max(-1)
        e = np.exp(s[:, a:b] - m[:, None])
        outs.append((e / e.sum(-1, keepdims=True)) @ v[a:b])
        maxs.append(m)
        sums.append(e.sum(-1))
    merged = attention.merge_blocks(np.stack(outs, 1), np.stack(maxs, 1), np.stack(sums, 1))
    assert np.allclose(merged, full, atol=1e-12)


def test_kv_row_quantizer_matches_reference_rule():
    """kv8.quantize_rows (kv8.py:39-43): s = max(max|x|/127, 1e-6), q = clip(rint(x/s))."""
    x = np.array([[0.0] * 4, [1.0, -2.0, 0.5, 127.0], [1e-9, -1e-9, 0, 0]], dtype=np.float32)
    q, s = kv.quantize_rows(x)
    assert s[0] == np.float32(1e-6) and np.all(q[0] == 0)
    assert s[1] == np.float32(1.0) and list(q[1]) == [1, -2, 0, 127]  # rint(0.5) = 0 (ties to even)
    assert s[2] == np.float32(1e-6)


def test_kv_g64_round_trip():
    rng = np.random.default_rng(10)
    x = rng.standard_normal((3, 256)).astype(np.float32)
    w, s, b = kv.quantize_g64(x)
    assert w.shape == (3, 64) and s.shape == (3, 4)
    back = kv.dequant_g64(w, s, b)
    step = np.repeat(bf16.bf16_bits_to_f32(s), 64, axis=-1)
    assert np.all(np.abs(back - x) <= 0.5 * step + 1e-2 * np.abs(x) + 1e-6)


# ---------------------------------------------------------------- fixtures

def test_golden_qmm_fixtures_regenerate():
    files = sorted(glob.glob(os.path.join(GOLDEN, "qmm_*.npz")))
    assert len(files) >= 5
    for f in files:
        g = load_golden(os.path.basename(f))
        assert np.array_equal(qmm.dequantize(g["w"], g["scales"], g["biases"]), g["deq"])
        y = qmm.qmm(g["x"], g["w"], g["scales"], g["biases"])
        assert np.allclose(y.astype(np.float32), g["y"], rtol=0, atol=1e-5)


def test_golden_attn_fixtures_regenerate():
    files = sorted(glob.glob(os.path.join(GOLDEN, "attn_*.npz")))
    assert len(files) >= 4
    for f in files:
        g = load_golden(os.path.basename(f))
        fmt = str(g["fmt"])
        if fmt == "bf16":
            kval, vval = bf16.bf16_bits_to_f32(g["k"]), bf16.bf16_bits_to_f32(g["v"])
        elif fmt == "ref_q8":
            kval, vval = kv.dequant_rows(g["k"], g["k_scale"]), kv.dequant_rows(g["v"], g["v_scale"])
        else:
            kval = kv.dequant_g64(g["k"], g["k_scales"], g["k_biases"])
            vval = kv.dequant_g64(g["v"], g["v_scales"], g["v_biases"])
        out = attention.tree_attention(bf16.bf16_bits_to_f32(g["q"]), kval, vval, int(g["n_kv"]), int(g["tail"]),
                                       g["bits"], float(g["scale"]))
        assert np.allclose(out, g["out"], atol=1e-5)


def test_decoder_oracle_rope_and_norm():
    """Self-checks of the decoder oracle (no GPU): rope is the identity at
    position 0 and leaves dims >= rope_dims alone, turns pair (i, i + dims/2)
    by pos * base^(-2i/dims); the RMS norm of a unit-weight row has unit RMS."""
    import numpy as np

    from oracle import decoder as od
    from oracle.bf16 import round_bf16

    rng = np.random.default_rng(0)
    x = rng.standard_normal((3, 256)).astype(np.float32)
    r = od.rope(x, np.array([5, 0, 100]), 64, 1e7)
    assert np.array_equal(r[1], round_bf16(x[1]))
    assert np.array_equal(r[:, 64:], round_bf16(x[:, 64:]))
    ang = 5 * 1e7 ** (-3 / 32)
    assert abs(r[0, 3] - (x[0, 3] * np.cos(ang) - x[0, 35] * np.sin(ang))) < 1e-2
    assert abs(r[0, 35] - (x[0, 3] * np.sin(ang) + x[0, 35] * np.cos(ang))) < 1e-2
    _, n = od.rms_norm(x, np.ones(256), 1e-6)
    assert np.allclose(np.sqrt(np.mean(n.astype(np.float64) ** 2, axis=-1)), 1, atol=1e-2)
    h, _ = od.rms_norm(x, np.ones(256), 1e-6, r=x)
    assert np.array_equal(h, round_bf16(2.0 * x.astype(np.float64)))


def test_decoder_oracle_gate_and_swiglu():
    import numpy as np

    from oracle import decoder as od

    gu = np.array([[0.0, 2.0, 3.0, -1.0]], dtype=np.float32)
    a = od.swiglu(gu)
    assert a[0, 0] == 0.0  # silu(0) = 0
    assert abs(a[0, 1] - 2.0 / (1 + np.exp(-2.0)) * -1.0) < 2e-2
    out = np.ones((1, 1, 1, 256), dtype=np.float32)
    g = np.zeros((1, 1, 256), dtype=np.float32)
    assert np.all(od.attn_gate(out, g) == 0.5)  # sigmoid(0) = 1/2


def test_take_rows_reads_before_writing():
    """oracle.kv.take_rows against a row loop that reads every kept row first
    (mx.take materialises the gather before the slice assignment,
    tree_verify.py:491-494), on a path that overlaps its destination."""
    from oracle import kv as okv

    rng = np.random.default_rng(3)
    t = rng.integers(-127, 128, size=(2, 3, 40, 16)).astype(np.int8)
    for start, nodes in [(4, [0, 2, 3, 9]), (0, [1, 2, 3]), (7, []), (10, list(range(12)))]:
        rows = [t[:, :, start + i].copy() for i in nodes]
        want = t.copy()
        for i, r in enumerate(rows):
            want[:, :, start + i] = r
        assert np.array_equal(okv.take_rows(t, start, nodes), want)
