"""The allocation-free attention entry point, tsb_tree_attn_noalloc.

It exists for callers that cannot allocate device memory on their decode
path (a pool-owned allocator, an FFI host without a device allocator, a
serving loop that forbids allocation): the split-KV scratch lives in a fixed
array inside the library instead of a caller workspace. These tests call it
through the C ABI and compare it with tsb_tree_attn given a workspace, on two
calls in a row with different inputs (the shared array keeps the previous
call's contents), and check that a call needing more scratch than the array
holds is refused before anything runs. This file is collected last, so a
failure here does not stop the rest of the suite."""

import ctypes

import numpy as np
import pytest
import torch

from gpu_util import assert_close_rel
from oracle import gen

pytestmark = pytest.mark.gpu

TSB_OK, TSB_EWORKSPACE = 0, 5


def _inputs(seed, bsz=1, t=16, hq=24, hkv=4, d=256, prefix=4096):
    g = torch.Generator(device="cuda").manual_seed(seed)
    n_kv = prefix + t
    q = torch.randn(bsz, hq, t, d, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(bsz, hkv, n_kv, d, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(bsz, hkv, n_kv, d, device="cuda", generator=g).to(torch.bfloat16)
    rng = np.random.default_rng(seed)
    parents = torch.from_numpy(np.stack([gen.tree_parents(rng, t) for _ in range(bsz)])).cuda()
    return q, k, v, parents, n_kv


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def test_noalloc_matches_workspace_entry_point_twice():
    import tsb
    from tsb import _lib

    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    for seed in (11, 12):  # two calls in a row, different inputs
        q, k, v, parents, n_kv = _inputs(seed)
        bsz, hq, t, d = q.shape
        hkv = k.shape[1]
        need = lib.tsb_tree_attn_workspace_bytes(bsz, t, hq, hkv, d, n_kv, tsb.TSB_KV_BF16)
        assert 0 < need <= 16 << 20  # the case exercises the library's scratch
        ws = torch.empty(need, dtype=torch.uint8, device="cuda")
        ref = torch.empty_like(q)
        ref_lse = torch.empty(bsz, hq, t, dtype=torch.float32, device="cuda")
        got = torch.full_like(q, float("nan"))
        got_lse = torch.full((bsz, hq, t), float("nan"), dtype=torch.float32, device="cuda")
        st = lib.tsb_tree_attn(_p(q), _p(k), None, None, _p(v), None, None, tsb.TSB_KV_BF16, _p(parents), None,
                               bsz, t, hq, hkv, d, n_kv, t, n_kv, d**-0.5, _p(ref), _p(ref_lse), _p(ws), need,
                               ctypes.c_void_p(stream))
        assert st == TSB_OK
        st = lib.tsb_tree_attn_noalloc(_p(q), _p(k), None, None, _p(v), None, None, tsb.TSB_KV_BF16, _p(parents),
                                       None, bsz, t, hq, hkv, d, n_kv, t, n_kv, d**-0.5, _p(got), _p(got_lse),
                                       ctypes.c_void_p(stream))
        assert st == TSB_OK
        torch.cuda.synchronize()
        assert_close_rel(got.float().cpu().numpy(), ref.float().cpu().numpy(), 2e-2, f"call seed {seed}")
        assert np.allclose(got_lse.cpu().numpy(), ref_lse.cpu().numpy(), atol=1e-2)
    assert lib.tsb_device_status(None, 0) == TSB_OK


def test_noalloc_refuses_more_than_its_scratch():
    import tsb
    from tsb import _lib

    lib = _lib.load()
    # 4 requests x 64 nodes x 32 query heads over 2 KV heads needs ~25 MB of partials
    bsz, t, hq, hkv, d, n_kv = 4, 64, 32, 2, 256, 4096
    need = lib.tsb_tree_attn_workspace_bytes(bsz, t, hq, hkv, d, n_kv, tsb.TSB_KV_BF16)
    assert need > 16 << 20
    out = torch.zeros(1, dtype=torch.bfloat16, device="cuda")
    st = lib.tsb_tree_attn_noalloc(None, None, None, None, None, None, None, tsb.TSB_KV_BF16, None, None,
                                   bsz, t, hq, hkv, d, n_kv, t, n_kv, d**-0.5, _p(out), None, None)
    assert st == TSB_EWORKSPACE
    assert b"workspace" in lib.tsb_strerror(st)
