"""Host-side logic of the tsb package (input makers, argument handling). No GPU."""

import numpy as np
import pytest
import torch

from oracle import bf16, kv, qmm


def test_torch_quantizer_matches_oracle():
    from tsb import quant

    rng = np.random.default_rng(11)
    w = (rng.standard_normal((64, 512)) * 0.02).astype(np.float32)
    w[3, :64] = 0.5  # a constant group
    wq, s, b = quant.quantize(torch.from_numpy(w))
    owq, os_, ob = qmm.quantize(w)
    assert np.array_equal(wq.numpy().view(np.uint32), owq)
    assert np.array_equal(bf16.from_torch_bf16(s), os_)
    assert np.array_equal(bf16.from_torch_bf16(b), ob)


def test_torch_kv_quantizers_match_oracle():
    from tsb import quant

    rng = np.random.default_rng(12)
    x = rng.standard_normal((2, 3, 5, 256)).astype(np.float32)
    q, s = quant.quantize_rows(torch.from_numpy(x))
    oq, os_ = kv.quantize_rows(x)
    assert np.array_equal(q.numpy(), oq) and np.array_equal(s.numpy(), os_)
    w, sc, bi = quant.quantize_g64(torch.from_numpy(x))
    ow, osc, obi = kv.quantize_g64(x)
    assert np.array_equal(w.numpy().view(np.uint32), ow)
    assert np.array_equal(bf16.from_torch_bf16(sc), osc) and np.array_equal(bf16.from_torch_bf16(bi), obi)


def test_pack_unpack_torch():
    from tsb import quant

    q = torch.randint(0, 16, (5, 64), dtype=torch.uint8)
    assert torch.equal(quant.unpack_bits(quant.pack_bits(q, 4), 4), q)
    assert np.array_equal(quant.pack_bits(q, 4).numpy().view(np.uint32), qmm.pack_bits(q.numpy(), 4))


def test_ops_refuse_cpu_tensors():
    """There is no CPU path: CPU tensors are rejected before any library call."""
    from tsb import ops

    x = torch.zeros(2, 128, dtype=torch.bfloat16)
    w = torch.zeros(128, 16, dtype=torch.int32)
    s = torch.zeros(128, 2, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.quantized_matmul(x, w, s, s)
    with pytest.raises(ValueError, match="CUDA"):
        ops.dequantize(w, s, s)


def test_kv_plane_selection():
    from tsb import ops
    from tsb.cache import KVCache, MLXQ8KVCache, Q8KVCache

    t = torch.zeros(1)
    assert ops._kv_planes(KVCache(t, t, 0))[0] == 0
    assert ops._kv_planes(Q8KVCache(t, t, t, t, 0))[0] == 2
    assert ops._kv_planes(MLXQ8KVCache(t, t, t, t, t, t, 0))[0] == 1

    class RefStyle:  # the reference's duck-typed cache: keys/values/offset (+ k_scale/v_scale)
        keys = values = t
        offset = 0
        k_scale = v_scale = t

    assert ops._kv_planes(RefStyle())[0] == 2
