"""Helpers for the GPU parity tests: numpy fixtures <-> torch CUDA tensors."""

import numpy as np
import torch

from oracle import bf16


def dev_bf16(bits):
    return bf16.to_torch_bf16(bits).cuda()


def dev_u32(w):
    return torch.from_numpy(np.ascontiguousarray(w).view(np.int32)).cuda()


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def host_bf16_bits(t):
    return bf16.from_torch_bf16(t)


def host_f32(t):
    return t.detach().float().cpu().numpy()


def assert_close_rel(got, ref, rel=2e-2, what=""):
    """max|got - ref| <= rel * max|ref| (the tolerance for bf16 outputs)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    err = np.max(np.abs(got - ref)) if ref.size else 0.0
    bound = rel * np.max(np.abs(ref)) if ref.size else 0.0
    assert err <= bound, f"{what}: max abs err {err:.4g} > {rel} * max|ref| = {bound:.4g}"
    return err
