"""The verify-step decoder (the gated-q layer stack) on the library's kernels.

One step runs every layer of a gated-q decoder over the tree nodes of B
requests (M = B*T rows), as mlx-tree-spec's batch_forward does
(src/mlx_tree_spec/tree_verify.py:414-447, attention 311-367, add_rms_norm
fused_ops.py:107-154):

    x = input_norm_0(h)
    per layer:  qkv = x W_qkv^T                     (4-bit qmm; q with gate, k, v)
                q, cache <- qkv_prep(qkv)            (q/k norms, rope at depth, K/V append)
                a = tree_attention(q, cache, parents)
                r = (a * sigmoid(gate)) W_o^T        (attn_gate + 4-bit qmm)
                h, x = add_rms_norm(h, r, post_norm)
                r = swiglu(x W_gate_up^T) W_down^T   (4-bit qmm, swiglu, 4-bit qmm)
                h, x = add_rms_norm(h, r, next input norm | final norm)

Per layer that is four quantized matmuls, one attention and five small
kernels; every buffer is allocated once per (B, T), so a whole step can be
captured in one CUDA graph (no host work inside). Weights are random (config 5
is a synthetic model): N(0, 0.02) quantized to 4-bit g64, norm weights
1 + N(0, 0.1). Rope follows a Qwen3-Next-style partial rotary layout (the
first `rope_dims` of each head, base `rope_base`); the reference reads both
from its model's config.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib, ops
from ._lib import TSB_KV_BF16, TSB_KV_MLX_Q8_G64, TSB_KV_REF_Q8_ROW, check
from .cache import KVCache, MLXQ8KVCache, Q8KVCache
from .quant import quantize, quantize_g64, quantize_rows


@dataclass
class DecoderConfig:
    layers: int = 16
    hidden: int = 5120
    hq: int = 24
    hkv: int = 4
    d: int = 256
    inter: int = 17408
    eps: float = 1e-6
    rope_dims: int = 64
    rope_base: float = 1e7

    @property
    def qkv_rows(self) -> int:
        return (2 * self.hq + 2 * self.hkv) * self.d


def random_weights(cfg: DecoderConfig, seed: int = 0, device="cuda", std: float = 0.02):
    """Per-layer weights {qkv, o, gate_up, down: (wq, scales, biases); q_norm,
    k_norm, input_norm, post_norm: bf16} and the final norm."""
    gen = torch.Generator(device=device).manual_seed(seed)

    def w(n, k):
        return quantize(torch.randn(n, k, generator=gen, device=device) * std)

    def norm(n):
        return (1.0 + 0.1 * torch.randn(n, generator=gen, device=device)).to(torch.bfloat16)

    layers = []
    for _ in range(cfg.layers):
        layers.append({"qkv": w(cfg.qkv_rows, cfg.hidden), "o": w(cfg.hidden, cfg.hq * cfg.d),
                       "gate_up": w(2 * cfg.inter, cfg.hidden), "down": w(cfg.hidden, cfg.inter),
                       "q_norm": norm(cfg.d), "k_norm": norm(cfg.d),
                       "input_norm": norm(cfg.hidden), "post_norm": norm(cfg.hidden)})
    return layers, norm(cfg.hidden)


def make_cache(kf: torch.Tensor, vf: torch.Tensor, offset: int, kv_format: int = TSB_KV_BF16):
    """A layer's cache from float K/V (B, Hkv, capacity, D) in the given format."""
    if kv_format == TSB_KV_BF16:
        return KVCache(kf.to(torch.bfloat16), vf.to(torch.bfloat16), offset)
    if kv_format == TSB_KV_REF_Q8_ROW:
        kq, ks = quantize_rows(kf)
        vq, vs = quantize_rows(vf)
        return Q8KVCache(kq, vq, ks, vs, offset)
    kw, ks, kb = quantize_g64(kf)
    vw, vs, vb = quantize_g64(vf)
    return MLXQ8KVCache(kw, vw, ks, kb, vs, vb, offset)


def _planes(cache):
    """(k, k_scales, k_biases, v, v_scales, v_biases) of a cache, as ops reads them."""
    fmt = cache.kv_format
    if fmt == TSB_KV_BF16:
        return cache.keys, None, None, cache.values, None, None
    if fmt == TSB_KV_REF_Q8_ROW:
        return cache.keys, cache.k_scale, None, cache.values, cache.v_scale, None
    return cache.keys, cache.k_scales, cache.k_biases, cache.values, cache.v_scales, cache.v_biases


def _ptr(t):
    return None if t is None else t.data_ptr()


class VerifyDecoder:
    """The layer stack over one verify step's nodes."""

    def __init__(self, cfg: DecoderConfig, layers, final_norm):
        self.cfg, self.layers, self.final_norm = cfg, layers, final_norm
        self._bufs: dict = {}

    def _buffers(self, b: int, t: int, device):
        key = (b, t, str(device))
        buf = self._bufs.get(key)
        if buf is None:
            c, m = self.cfg, b * t
            e = lambda *shape, dt=torch.bfloat16: torch.empty(*shape, dtype=dt, device=device)  # noqa: E731
            buf = {"h": e(m, c.hidden), "x": e(m, c.hidden), "r": e(m, c.hidden), "qkv": e(m, c.qkv_rows),
                   "q": e(b, c.hq, t, c.d), "attn": e(b, c.hq, t, c.d), "gated": e(m, c.hq * c.d),
                   "gu": e(m, 2 * c.inter), "act": e(m, c.inter),
                   "positions": e(m, dt=torch.int32), "offsets": e(b, dt=torch.int32)}
            self._bufs[key] = buf
        return buf

    def step(self, h_in: torch.Tensor, parents: torch.Tensor, caches, prefix: int) -> torch.Tensor:
        """h_in (B*T, hidden) bf16 hidden states of the nodes (request-major);
        parents int32 (B, T); caches: one per layer, holding `prefix` rows per
        request and room for T more (their offset is set to prefix + T). The
        nodes' K/V are written at rows prefix .. prefix+T-1. Returns the final
        normed hidden states (B*T, hidden), a buffer reused by the next step."""
        c = self.cfg
        b, t = parents.shape
        m = b * t
        dev = h_in.device
        buf = self._buffers(b, t, dev)
        lib = _lib.load()
        st = torch.cuda.current_stream(dev).cuda_stream
        _, depth = ops.ancestor_bits(parents, depth=True)
        buf["positions"].copy_((depth + prefix).reshape(-1))
        buf["offsets"].fill_(prefix)
        h, x, r = buf["h"], buf["x"], buf["r"]
        h.copy_(h_in)
        check(lib.tsb_add_rms_norm(_ptr(h), None, _ptr(self.layers[0]["input_norm"]), None, _ptr(x), m, c.hidden,
                                   c.eps, st), "tsb_add_rms_norm")
        scale = c.d ** -0.5
        for i, lw in enumerate(self.layers):
            cache = caches[i]
            cache.offset = prefix + t
            k, ks, kb, v, vs, vb = _planes(cache)
            ops.quantized_matmul_into(x, *lw["qkv"], buf["qkv"], c.qkv_rows)
            check(lib.tsb_qkv_prep(_ptr(buf["qkv"]), c.qkv_rows, b, t, c.hq, c.hkv, c.d, _ptr(lw["q_norm"]),
                                   _ptr(lw["k_norm"]), c.eps, _ptr(buf["positions"]), c.rope_dims, c.rope_base, 1.0,
                                   _ptr(buf["q"]), cache.kv_format, _ptr(k), _ptr(ks), _ptr(kb), _ptr(v), _ptr(vs),
                                   _ptr(vb), k.shape[2], _ptr(buf["offsets"]), st), "tsb_qkv_prep")
            if ops.tree_flash(buf["q"], cache, scale, parents=parents, out=buf["attn"]) is None:
                raise RuntimeError("tree attention declined the decoder's shape")
            check(lib.tsb_attn_gate(_ptr(buf["attn"]), _ptr(buf["qkv"]), c.qkv_rows, _ptr(buf["gated"]), b, t, c.hq,
                                    c.d, st), "tsb_attn_gate")
            ops.quantized_matmul_into(buf["gated"], *lw["o"], r, c.hidden)
            check(lib.tsb_add_rms_norm(_ptr(h), _ptr(r), _ptr(lw["post_norm"]), _ptr(h), _ptr(x), m, c.hidden, c.eps,
                                       st), "tsb_add_rms_norm")
            ops.quantized_matmul_into(x, *lw["gate_up"], buf["gu"], 2 * c.inter)
            check(lib.tsb_swiglu(_ptr(buf["gu"]), _ptr(buf["act"]), m, c.inter, st), "tsb_swiglu")
            ops.quantized_matmul_into(buf["act"], *lw["down"], r, c.hidden)
            nxt = self.layers[i + 1]["input_norm"] if i + 1 < len(self.layers) else self.final_norm
            check(lib.tsb_add_rms_norm(_ptr(h), _ptr(r), _ptr(nxt), _ptr(h), _ptr(x), m, c.hidden, c.eps, st),
                  "tsb_add_rms_norm")
        return x


__all__ = ["DecoderConfig", "random_weights", "make_cache", "VerifyDecoder",
           "TSB_KV_BF16", "TSB_KV_MLX_Q8_G64", "TSB_KV_REF_Q8_ROW"]
