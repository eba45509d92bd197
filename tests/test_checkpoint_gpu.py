"""The MLX checkpoint loader feeding the verify-step decoder on the GPU: a
decoder's weights written as an mlx-lm checkpoint (separate q/k/v and
gate/up projections, two safetensors shards) load back into HBM bit-exact,
fused as the decoder wants them, and one decoder step over the loaded weights
equals the step over the originals bit for bit."""

import pytest
import torch

from ckpt_util import decoder_config_json, decoder_tensors, write_checkpoint

pytestmark = pytest.mark.gpu


def test_loaded_decoder_matches(tmp_path):
    import tsb
    from tsb import decoder as tdec
    from tsb.checkpoint import Checkpoint, decoder_config, decoder_layers

    cfg = tdec.DecoderConfig(layers=2, hidden=1024, hq=4, hkv=1, d=256, inter=1024)
    layers, final_norm = tdec.random_weights(cfg, seed=7)
    write_checkpoint(str(tmp_path), decoder_tensors(cfg, layers, final_norm), decoder_config_json(cfg))
    ck = Checkpoint(str(tmp_path))
    lcfg = decoder_config(ck)
    assert lcfg == cfg
    got_layers, got_norm = decoder_layers(ck, lcfg, device="cuda")
    assert len(got_layers) == cfg.layers
    for a, b in zip(layers, got_layers):
        for key in ("qkv", "o", "gate_up", "down"):
            for x, y in zip(a[key], b[key]):
                assert x.dtype == y.dtype and x.shape == y.shape and torch.equal(x.view(torch.int16), y.view(torch.int16))
        for key in ("q_norm", "k_norm", "input_norm", "post_norm"):
            assert torch.equal(a[key].view(torch.int16), b[key].view(torch.int16))
    assert torch.equal(final_norm.view(torch.int16), got_norm.view(torch.int16))

    b, t, prefix = 2, 8, 100
    cap = prefix + t
    g = torch.Generator(device="cuda").manual_seed(3)
    kf = [torch.randn(b, cfg.hkv, cap, 256, device="cuda", generator=g) for _ in range(cfg.layers)]
    vf = [torch.randn(b, cfg.hkv, cap, 256, device="cuda", generator=g) for _ in range(cfg.layers)]
    parents = torch.tensor([[-1, 0, 0, 1, 1, 2, 3, 6], [-1, 0, 1, 2, 3, 4, 5, 6]], dtype=torch.int32, device="cuda")
    h0 = torch.randn(b * t, cfg.hidden, device="cuda", generator=g).to(torch.bfloat16)
    outs = []
    for lw, fn in ((layers, final_norm), (got_layers, got_norm)):
        caches = [tdec.make_cache(kf[i], vf[i], prefix, tsb.TSB_KV_BF16) for i in range(cfg.layers)]
        outs.append(tdec.VerifyDecoder(cfg, lw, fn).step(h0, parents, caches, prefix).clone())
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
