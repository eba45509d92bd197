"""The verify-step decoder's kernels and a small decoder step against the CPU
oracle (oracle/decoder.py).

Bars: the 8-bit appends are bit-exact against the oracle's quantizers applied
to the kernel's own bf16 rows; the other outputs within 1e-2 * max|ref| per
op (bf16 rounding of values computed with float32 rsqrt/exp/sincos), and the
decoder step's output within 2e-2 * max|ref|."""

import numpy as np
import pytest
import torch

from gpu_util import assert_close_rel, host_f32
from oracle import bf16 as obf16
from oracle import decoder as odec
from oracle import gen, kv, tree

pytestmark = pytest.mark.gpu


def _lib():
    import tsb

    return tsb._lib.load()


def _st():
    return torch.cuda.current_stream().cuda_stream


def _bf(t):
    return obf16.from_torch_bf16(t.cpu())


def _w_np(w):
    wq, s, b = w
    return wq.cpu().numpy().view(np.uint32), _bf(s), _bf(b)


@pytest.mark.parametrize("rows,d,residual", [(16, 5120, True), (128, 5120, False), (3, 1024, True)])
def test_add_rms_norm(rows, d, residual):
    g = torch.Generator(device="cuda").manual_seed(rows + d)
    x = torch.randn(rows, d, device="cuda", generator=g).to(torch.bfloat16)
    r = torch.randn(rows, d, device="cuda", generator=g).to(torch.bfloat16) if residual else None
    w = (1 + 0.1 * torch.randn(d, device="cuda", generator=g)).to(torch.bfloat16)
    h = torch.empty_like(x)
    n = torch.empty_like(x)
    st = _lib().tsb_add_rms_norm(x.data_ptr(), r.data_ptr() if residual else None, w.data_ptr(),
                                 h.data_ptr() if residual else None, n.data_ptr(), rows, d, 1e-6, _st())
    assert st == 0
    torch.cuda.synchronize()
    h_ref, n_ref = odec.rms_norm(host_f32(x), host_f32(w), 1e-6, host_f32(r) if residual else None)
    if residual:
        assert np.array_equal(host_f32(h), h_ref)  # bf16(x + r): exact
    assert_close_rel(host_f32(n), n_ref, 1e-2, "norm")


def _prep_inputs(b, t, hq, hkv, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    ld = (2 * hq + 2 * hkv) * 256
    qkv = torch.randn(b * t, ld, device="cuda", generator=g).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(256, device="cuda", generator=g)).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(256, device="cuda", generator=g)).to(torch.bfloat16)
    rng = np.random.default_rng(seed)
    parents = np.stack([gen.tree_parents(rng, t) for _ in range(b)])
    prefix = 1000 + 37 * seed % 500
    pos = (np.stack([tree.depth(p) for p in parents]) + prefix).astype(np.int32).reshape(-1)
    return qkv, qn, kn, parents, prefix, pos


def _run_prep(qkv, qn, kn, pos, b, t, hq, hkv, cap, prefix, fmt, rope_dims=64, rope_base=1e7):
    import tsb

    dev = "cuda"
    q_out = torch.empty(b, hq, t, 256, dtype=torch.bfloat16, device=dev)
    if fmt == tsb.TSB_KV_BF16:
        k = torch.zeros(b, hkv, cap, 256, dtype=torch.bfloat16, device=dev)
        v = torch.zeros_like(k)
        aux = [None] * 4
    elif fmt == tsb.TSB_KV_REF_Q8_ROW:
        k = torch.zeros(b, hkv, cap, 256, dtype=torch.int8, device=dev)
        v = torch.zeros_like(k)
        aux = [torch.zeros(b, hkv, cap, device=dev), None, torch.zeros(b, hkv, cap, device=dev), None]
    else:
        k = torch.zeros(b, hkv, cap, 64, dtype=torch.int32, device=dev)
        v = torch.zeros_like(k)
        aux = [torch.zeros(b, hkv, cap, 4, dtype=torch.bfloat16, device=dev) for _ in range(4)]
    posd = torch.from_numpy(pos).cuda()
    offs = torch.full((b,), prefix, dtype=torch.int32, device=dev)
    p = lambda a: None if a is None else a.data_ptr()  # noqa: E731
    st = _lib().tsb_qkv_prep(qkv.data_ptr(), qkv.shape[1], b, t, hq, hkv, 256, qn.data_ptr(), kn.data_ptr(), 1e-6,
                             posd.data_ptr(), rope_dims, rope_base, 1.0, q_out.data_ptr(), fmt, k.data_ptr(),
                             p(aux[0]), p(aux[1]), v.data_ptr(), p(aux[2]), p(aux[3]), cap, offs.data_ptr(), _st())
    assert st == 0
    torch.cuda.synchronize()
    return q_out, k, v, aux


@pytest.mark.parametrize("b,t,hq,hkv,rope_dims", [(4, 32, 24, 4, 64), (2, 5, 8, 2, 256), (1, 3, 4, 1, 16)])
def test_qkv_prep_bf16(b, t, hq, hkv, rope_dims):
    import tsb

    qkv, qn, kn, parents, prefix, pos = _prep_inputs(b, t, hq, hkv, seed=b + t)
    cap = prefix + t + 3
    q_out, k, v, _ = _run_prep(qkv, qn, kn, pos, b, t, hq, hkv, cap, prefix, tsb.TSB_KV_BF16, rope_dims=rope_dims)
    q_ref, k_ref, v_ref, _ = odec.qkv_prep(host_f32(qkv), hq, hkv, host_f32(qn), host_f32(kn), 1e-6, pos, b, t,
                                          rope_dims, 1e7)
    assert_close_rel(host_f32(q_out), q_ref, 1e-2, "queries")
    kk = host_f32(k)
    assert_close_rel(kk[:, :, prefix:prefix + t], k_ref, 1e-2, "keys")
    assert np.array_equal(host_f32(v)[:, :, prefix:prefix + t], v_ref)  # values copied as they are
    # nothing outside the nodes' rows was written
    assert not kk[:, :, :prefix].any() and not kk[:, :, prefix + t:].any()


@pytest.mark.parametrize("fmt", ["mlx_q8", "ref_q8"])
def test_qkv_prep_quantize_on_append_bit_exact(fmt):
    """The 8-bit append equals the oracle quantizer applied to the kernel's own
    bf16 key/value rows (same kernel, bf16 cache)."""
    import tsb

    b, t, hq, hkv = 2, 8, 8, 2
    qkv, qn, kn, parents, prefix, pos = _prep_inputs(b, t, hq, hkv, seed=11)
    cap = prefix + t
    _, kb, vb, _ = _run_prep(qkv, qn, kn, pos, b, t, hq, hkv, cap, prefix, tsb.TSB_KV_BF16)
    code = tsb.TSB_KV_MLX_Q8_G64 if fmt == "mlx_q8" else tsb.TSB_KV_REF_Q8_ROW
    _, kq, vq, aux = _run_prep(qkv, qn, kn, pos, b, t, hq, hkv, cap, prefix, code)
    for rows_bf16, codes, sc, bi in ((kb, kq, aux[0], aux[1]), (vb, vq, aux[2], aux[3])):
        x = host_f32(rows_bf16)[:, :, prefix:prefix + t]
        if fmt == "mlx_q8":
            w_ref, s_ref, b_ref = kv.quantize_g64(x)
            assert np.array_equal(codes.cpu().numpy().view(np.uint32)[:, :, prefix:prefix + t], w_ref)
            assert np.array_equal(_bf(sc)[:, :, prefix:prefix + t], s_ref)
            assert np.array_equal(_bf(bi)[:, :, prefix:prefix + t], b_ref)
        else:
            q_ref, s_ref = kv.quantize_rows(x)
            assert np.array_equal(codes.cpu().numpy()[:, :, prefix:prefix + t], q_ref)
            assert np.array_equal(sc.cpu().numpy()[:, :, prefix:prefix + t], s_ref)


def test_attn_gate_and_swiglu():
    b, t, hq, inter = 4, 32, 24, 17408
    g = torch.Generator(device="cuda").manual_seed(3)
    out = torch.randn(b, hq, t, 256, device="cuda", generator=g).to(torch.bfloat16)
    qkv = torch.randn(b * t, (2 * hq + 8) * 256, device="cuda", generator=g).to(torch.bfloat16)
    y = torch.empty(b * t, hq * 256, dtype=torch.bfloat16, device="cuda")
    assert _lib().tsb_attn_gate(out.data_ptr(), qkv.data_ptr(), qkv.shape[1], y.data_ptr(), b, t, hq, 256, _st()) == 0
    gu = torch.randn(b * t, 2 * inter, device="cuda", generator=g).to(torch.bfloat16)
    a = torch.empty(b * t, inter, dtype=torch.bfloat16, device="cuda")
    assert _lib().tsb_swiglu(gu.data_ptr(), a.data_ptr(), b * t, inter, _st()) == 0
    torch.cuda.synchronize()
    gate = host_f32(qkv)[:, :hq * 512].reshape(b * t, hq, 512)[..., 256:]
    assert_close_rel(host_f32(y), odec.attn_gate(host_f32(out), gate), 1e-2, "gate")
    assert_close_rel(host_f32(a), odec.swiglu(host_f32(gu)), 1e-2, "swiglu")


@pytest.mark.parametrize("fmt", ["bf16", "mlx_q8"])
def test_decoder_step_small(fmt):
    """Two layers (hidden 1024, 4q/1kv heads of 256, MLP 1024), 2 requests x 8
    nodes over a 200-row prefix, against the oracle's layer loop."""
    import tsb
    from tsb import decoder as tdec

    cfg = tdec.DecoderConfig(layers=2, hidden=1024, hq=4, hkv=1, d=256, inter=1024)
    layers, final_norm = tdec.random_weights(cfg, seed=5)
    b, t, prefix = 2, 8, 200
    cap = prefix + t + 8
    g = torch.Generator(device="cuda").manual_seed(9)
    code = tsb.TSB_KV_BF16 if fmt == "bf16" else tsb.TSB_KV_MLX_Q8_G64
    kf = [torch.randn(b, cfg.hkv, cap, 256, device="cuda", generator=g) for _ in range(cfg.layers)]
    vf = [torch.randn(b, cfg.hkv, cap, 256, device="cuda", generator=g) for _ in range(cfg.layers)]
    caches = [tdec.make_cache(kf[i], vf[i], prefix, code) for i in range(cfg.layers)]
    # the oracle's prefix: the values the GPU cache holds
    if fmt == "bf16":
        kref = [host_f32(c.keys).astype(np.float64) for c in caches]
        vref = [host_f32(c.values).astype(np.float64) for c in caches]
    else:
        kref = [kv.dequant_g64(c.keys.cpu().numpy().view(np.uint32), _bf(c.k_scales), _bf(c.k_biases)) for c in caches]
        vref = [kv.dequant_g64(c.values.cpu().numpy().view(np.uint32), _bf(c.v_scales), _bf(c.v_biases))
                for c in caches]
    rng = np.random.default_rng(4)
    parents = np.stack([gen.tree_parents(rng, t) for _ in range(b)]).astype(np.int32)
    h0 = torch.randn(b * t, cfg.hidden, device="cuda", generator=g).to(torch.bfloat16)
    dec = tdec.VerifyDecoder(cfg, layers, final_norm)
    out = dec.step(h0, torch.from_numpy(parents).cuda(), caches, prefix)
    torch.cuda.synchronize()
    got = host_f32(out)
    # oracle
    ocfg = {"hq": cfg.hq, "hkv": cfg.hkv, "d": cfg.d, "eps": cfg.eps, "rope_dims": cfg.rope_dims,
            "rope_base": cfg.rope_base}
    h = host_f32(h0)
    _, x = odec.rms_norm(h, host_f32(layers[0]["input_norm"]), cfg.eps)
    for i, lw in enumerate(layers):
        p = {name: _w_np(lw[name]) for name in ("qkv", "o", "gate_up", "down")}
        p.update({name: host_f32(lw[name]) for name in ("q_norm", "k_norm", "post_norm")})
        nxt = host_f32(layers[i + 1]["input_norm"]) if i + 1 < len(layers) else host_f32(final_norm)
        # the nodes' rows go into the cache in its format (quantized on append)
        h, x = odec.layer_step(h, x, p, kref[i], vref[i], parents, [prefix] * b, ocfg, nxt, kv_format=fmt)
    assert_close_rel(got, x, 2e-2, f"decoder {fmt}")
