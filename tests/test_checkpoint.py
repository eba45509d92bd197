"""The MLX checkpoint loader (tsb.checkpoint) on the CPU: the safetensors
parser against files written by the `safetensors` package, the eligibility
rule (mlx-tree-spec src/mlx_tree_spec/packed_linear.py:49-58 plus this
library's group-64 / bf16 / N % 128 limits), mlx-lm's per-module quantization
overrides, fused row concatenation and per-rank row shards, all bit-exact."""

import json
import os

import numpy as np
import pytest
import torch

from ckpt_util import write_checkpoint
from oracle import gen


def _w(rng, n, k):
    wq, s, b = gen.weights_w4g64(rng, n, k)
    return (torch.from_numpy(wq.view(np.int32)), torch.from_numpy(s.view(np.int16)).view(torch.bfloat16),
            torch.from_numpy(b.view(np.int16)).view(torch.bfloat16))


def _bits(t):
    t = t.cpu()
    return t.view(torch.int16).numpy() if t.dtype in (torch.bfloat16, torch.float16) else t.numpy()


@pytest.fixture(scope="module")
def ckpt_dir(tmp_path_factory):
    rng = np.random.default_rng(0)
    mods = {"m.q": (640, 256), "m.k": (256, 256), "m.v": (128, 256), "m.o": (256, 512), "m.narrow": (96, 256),
            "m.q8": (128, 256), "m.fp16": (128, 256), "m.biased": (128, 256), "m.plain": (128, 256)}
    tensors, w = {}, {}
    for name, (n, k) in mods.items():
        w[name] = _w(rng, n, k)
        for part, t in zip(("weight", "scales", "biases"), w[name]):
            tensors[f"{name}.{part}"] = t
    tensors["m.fp16.scales"] = tensors["m.fp16.scales"].float().to(torch.float16)
    tensors["m.biased.bias"] = torch.zeros(128, dtype=torch.bfloat16)
    tensors["m.norm.weight"] = torch.randn(256).to(torch.bfloat16)
    tensors["m.f32"] = torch.randn(3, 5)
    cfg = {"quantization": {"group_size": 64, "bits": 4, "m.q8": {"bits": 8, "group_size": 64}, "m.plain": False}}
    path = str(tmp_path_factory.mktemp("ckpt"))
    write_checkpoint(path, tensors, cfg, n_files=3)
    return path, tensors, w


def test_header_matches_writer(ckpt_dir):
    from tsb.checkpoint import Checkpoint

    path, tensors, _ = ckpt_dir
    ck = Checkpoint(path)
    assert set(ck.tensors) == set(tensors)
    for name, t in tensors.items():
        e = ck.tensors[name]
        assert e.shape == tuple(t.shape)
        got = ck.load_tensor(name, "cpu")
        assert np.array_equal(_bits(got), _bits(t if t.dtype != torch.uint32 else t.view(torch.int32))), name


def test_eligibility(ckpt_dir):
    from tsb.checkpoint import Checkpoint

    ck = Checkpoint(ckpt_dir[0])
    reasons = ck.quantized_linears()
    for m in ("m.q", "m.k", "m.v", "m.o"):
        assert reasons[m] is None, (m, reasons[m])
    assert "128 rows" in reasons["m.narrow"]     # N=96 passes the reference's rule, not the 128-row tiles
    assert "8-bit" in reasons["m.q8"]            # per-module override
    assert "bf16" in reasons["m.fp16"]
    assert "bias" in reasons["m.biased"]
    assert reasons["m.plain"] == "not quantized"  # override false
    with pytest.raises(ValueError):
        ck.load_linear("m.q8", "cpu")


def test_fused_and_sharded_rows(ckpt_dir):
    from tsb.checkpoint import Checkpoint

    path, _, w = ckpt_dir
    ck = Checkpoint(path)
    full = ck.load_linear(["m.q", "m.k", "m.v"], "cpu")
    want = [torch.cat([w[m][i] for m in ("m.q", "m.k", "m.v")]) for i in range(3)]
    for g, t in zip(full, want):
        assert np.array_equal(_bits(g), _bits(t))
    for world in (2, 4):
        parts = [ck.load_linear(["m.q", "m.k", "m.v"], "cpu", world=world, rank=r) for r in range(world)]
        for i in range(3):
            assert np.array_equal(_bits(torch.cat([p[i] for p in parts])), _bits(want[i]))
    with pytest.raises(ValueError):
        ck.load_linear(["m.q", "m.o"], "cpu")      # different K
    with pytest.raises(ValueError):
        ck.load_linear("m.v", "cpu", world=2, rank=0)   # 64-row shards are not on the fast path


def test_malformed_files(tmp_path):
    from tsb.checkpoint import read_header

    p = tmp_path / "bad.safetensors"
    head = json.dumps({"x": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]}}).encode()
    p.write_bytes(len(head).to_bytes(8, "little") + head + b"\0" * 8)    # 8 of the 16 data bytes
    with pytest.raises(ValueError):
        read_header(str(p))
    p.write_bytes((1 << 40).to_bytes(8, "little") + b"{}")
    with pytest.raises(ValueError):
        read_header(str(p))
    head = json.dumps({"x": {"dtype": "F32", "shape": [4], "data_offsets": [0, 12]}}).encode()
    p.write_bytes(len(head).to_bytes(8, "little") + head + b"\0" * 16)   # offsets disagree with the shape
    with pytest.raises(ValueError):
        read_header(str(p))


def test_decoder_config(tmp_path):
    from tsb.checkpoint import Checkpoint, decoder_config

    cfg = {"text_config": {"num_hidden_layers": 48, "hidden_size": 5120, "num_attention_heads": 24,
                           "num_key_value_heads": 4, "head_dim": 256, "intermediate_size": 17408,
                           "rms_norm_eps": 1e-6, "partial_rotary_factor": 0.25, "rope_theta": 1e7}}
    write_checkpoint(str(tmp_path), {"a": torch.zeros(1)}, cfg, n_files=1)
    c = decoder_config(Checkpoint(str(tmp_path)))
    assert (c.layers, c.hidden, c.hq, c.hkv, c.d, c.inter, c.rope_dims, c.rope_base) == \
        (48, 5120, 24, 4, 256, 17408, 64, 1e7)
    assert os.path.exists(tmp_path / "model.safetensors.index.json")


@pytest.mark.parametrize("where", ["top", "nested", "missing"])
def test_decoder_config_rope_layouts(tmp_path, where):
    """rope_theta / partial_rotary_factor at the top level or nested under
    "rope_parameters" (newer configs); a config without rope_theta is refused
    rather than given a default base."""
    from tsb.checkpoint import Checkpoint, decoder_config

    c = {"num_hidden_layers": 4, "hidden_size": 5120, "num_attention_heads": 24, "num_key_value_heads": 4,
         "head_dim": 256, "intermediate_size": 17408, "rms_norm_eps": 1e-6}
    rope = {"partial_rotary_factor": 0.25, "rope_theta": 1e7}
    if where == "top":
        c.update(rope)
    elif where == "nested":
        c["rope_parameters"] = dict(rope, rope_type="default")
    write_checkpoint(str(tmp_path), {"a": torch.zeros(1)}, {"text_config": c}, n_files=1)
    ck = Checkpoint(str(tmp_path))
    if where == "missing":
        with pytest.raises(ValueError):
            decoder_config(ck)
        assert decoder_config(ck, rope_base=5e6).rope_base == 5e6
        return
    cfg = decoder_config(ck)
    assert (cfg.rope_dims, cfg.rope_base) == (64, 1e7)


def test_decoder_layers_fuse_on_cpu(tmp_path):
    """decoder_layers reads an mlx-lm layout (separate q/k/v and gate/up) back
    into the decoder's fused projections, bit-exact, with the config's shapes."""
    from ckpt_util import decoder_config_json, decoder_tensors
    from tsb.checkpoint import Checkpoint, decoder_config, decoder_layers
    from tsb.decoder import DecoderConfig

    cfg = DecoderConfig(layers=2, hidden=256, hq=2, hkv=1, d=256, inter=256)
    rng = np.random.default_rng(5)
    norm = lambda n: torch.from_numpy(rng.standard_normal(n).astype(np.float32)).to(torch.bfloat16)  # noqa: E731
    layers = [{"qkv": _w(rng, cfg.qkv_rows, cfg.hidden), "o": _w(rng, cfg.hidden, cfg.hq * cfg.d),
               "gate_up": _w(rng, 2 * cfg.inter, cfg.hidden), "down": _w(rng, cfg.hidden, cfg.inter),
               "q_norm": norm(cfg.d), "k_norm": norm(cfg.d), "input_norm": norm(cfg.hidden),
               "post_norm": norm(cfg.hidden)} for _ in range(cfg.layers)]
    final = norm(cfg.hidden)
    write_checkpoint(str(tmp_path), decoder_tensors(cfg, layers, final), decoder_config_json(cfg))
    ck = Checkpoint(str(tmp_path))
    assert decoder_config(ck) == cfg
    got, got_final = decoder_layers(ck, cfg, device="cpu")
    for a, b in zip(layers, got):
        for key in ("qkv", "o", "gate_up", "down"):
            for x, y in zip(a[key], b[key]):
                assert np.array_equal(_bits(x), _bits(y)), key
        for key in ("q_norm", "k_norm", "input_norm", "post_norm"):
            assert np.array_equal(_bits(a[key]), _bits(b[key])), key
    assert np.array_equal(_bits(final), _bits(got_final))
    with pytest.raises(ValueError):
        decoder_layers(ck, DecoderConfig(layers=2, hidden=256, hq=4, hkv=1, d=256, inter=256), device="cpu")


def test_decoder_layers_find_the_language_model_prefix(tmp_path):
    """Multimodal mlx-lm checkpoints keep the text layers under
    language_model.model.layers (and the final norm beside them): found without
    naming the prefix; a checkpoint with no q_proj anywhere is refused."""
    from ckpt_util import decoder_config_json, decoder_tensors
    from tsb.checkpoint import Checkpoint, decoder_layers
    from tsb.decoder import DecoderConfig

    cfg = DecoderConfig(layers=1, hidden=256, hq=2, hkv=1, d=256, inter=256)
    rng = np.random.default_rng(6)
    norm = lambda n: torch.from_numpy(rng.standard_normal(n).astype(np.float32)).to(torch.bfloat16)  # noqa: E731
    layers = [{"qkv": _w(rng, cfg.qkv_rows, cfg.hidden), "o": _w(rng, cfg.hidden, cfg.hq * cfg.d),
               "gate_up": _w(rng, 2 * cfg.inter, cfg.hidden), "down": _w(rng, cfg.hidden, cfg.inter),
               "q_norm": norm(cfg.d), "k_norm": norm(cfg.d), "input_norm": norm(cfg.hidden),
               "post_norm": norm(cfg.hidden)}]
    final = norm(cfg.hidden)
    write_checkpoint(str(tmp_path / "mm"), decoder_tensors(cfg, layers, final, prefix="language_model.model.layers"),
                     decoder_config_json(cfg))
    got, got_final = decoder_layers(Checkpoint(str(tmp_path / "mm")), cfg, device="cpu")
    assert len(got) == 1 and np.array_equal(_bits(final), _bits(got_final))
    write_checkpoint(str(tmp_path / "none"), {"model.norm.weight": final}, decoder_config_json(cfg), n_files=1)
    with pytest.raises(ValueError):
        decoder_layers(Checkpoint(str(tmp_path / "none")), cfg, device="cpu")
