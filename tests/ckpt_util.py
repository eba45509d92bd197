"""Writes small mlx-lm-style checkpoints for the loader tests: safetensors
files written by the `safetensors` package (the format's own implementation,
so the loader's parser is checked against it), an index and a config.json."""

from __future__ import annotations

import json
import os

import torch


def as_stored(t: torch.Tensor) -> torch.Tensor:
    """int32 weight words are stored as MLX stores them: uint32."""
    t = t.detach().cpu().contiguous()
    return t.view(torch.uint32) if t.dtype == torch.int32 else t


def write_checkpoint(path: str, tensors: dict, config: dict, n_files: int = 2) -> None:
    """tensors {name: torch tensor} split round-robin over n_files shards."""
    from safetensors.torch import save_file

    os.makedirs(path, exist_ok=True)
    names = sorted(tensors)
    weight_map = {}
    for f in range(n_files):
        fname = f"model-{f + 1:05d}-of-{n_files:05d}.safetensors"
        part = {n: as_stored(tensors[n]) for n in names[f::n_files]}
        save_file(part, os.path.join(path, fname), metadata={"format": "mlx"})
        weight_map.update({n: fname for n in part})
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as fh:
        json.dump({"metadata": {}, "weight_map": weight_map}, fh)
    with open(os.path.join(path, "config.json"), "w") as fh:
        json.dump(config, fh)


def decoder_tensors(cfg, layers, final_norm, prefix: str = "model.layers") -> dict:
    """A VerifyDecoder weight set as an mlx-lm checkpoint's tensors: the fused
    qkv split back into q_proj (query|gate per head), k_proj, v_proj, gate_up
    into gate_proj and up_proj."""
    out = {}
    q_rows, kv_rows = 2 * cfg.hq * cfg.d, cfg.hkv * cfg.d
    for i, lw in enumerate(layers):
        p = f"{prefix}.{i}."

        def put(name, w, r0=0, r1=None):
            for part, t in zip(("weight", "scales", "biases"), w):
                out[f"{p}{name}.{part}"] = t[r0:r1]

        put("self_attn.q_proj", lw["qkv"], 0, q_rows)
        put("self_attn.k_proj", lw["qkv"], q_rows, q_rows + kv_rows)
        put("self_attn.v_proj", lw["qkv"], q_rows + kv_rows, None)
        put("self_attn.o_proj", lw["o"])
        put("mlp.gate_proj", lw["gate_up"], 0, cfg.inter)
        put("mlp.up_proj", lw["gate_up"], cfg.inter, None)
        put("mlp.down_proj", lw["down"])
        for key, name in (("q_norm", "self_attn.q_norm"), ("k_norm", "self_attn.k_norm"),
                          ("input_norm", "input_layernorm"), ("post_norm", "post_attention_layernorm")):
            out[f"{p}{name}.weight"] = lw[key]
    out[prefix[: -len(".layers")] + ".norm.weight"] = final_norm
    return out


def decoder_config_json(cfg) -> dict:
    return {"model_type": "qwen3_next", "num_hidden_layers": cfg.layers, "hidden_size": cfg.hidden,
            "num_attention_heads": cfg.hq, "num_key_value_heads": cfg.hkv, "head_dim": cfg.d,
            "intermediate_size": cfg.inter, "rms_norm_eps": cfg.eps,
            "partial_rotary_factor": cfg.rope_dims / cfg.d, "rope_theta": cfg.rope_base,
            "quantization": {"group_size": 64, "bits": 4, "mode": "affine"}}
