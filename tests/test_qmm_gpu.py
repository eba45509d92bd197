"""GPU parity of the quantized matmul and dequantization against the oracle.

Bar: dequantization bit-exact; qmm max-abs-err <= 2e-2 * max|ref| (bf16
output, fp32 accumulation), the tolerance of the verify path; the kernel is
also held to a much tighter bound against the exact result, since bf16
rounding of the output alone is ~0.4%."""

import glob
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, load_golden
from gpu_util import assert_close_rel, dev_bf16, dev_u32, host_bf16_bits, host_f32
from oracle import bf16, gen, qmm

pytestmark = pytest.mark.gpu

REL = 2e-2      # the verify path's tolerance
REL_TIGHT = 8e-3


def _run(x_bits, wq, s, b, out=None):
    import tsb

    y = tsb.quantized_matmul(dev_bf16(x_bits), dev_u32(wq), dev_bf16(s), dev_bf16(b))
    torch.cuda.synchronize()
    assert y is not None
    return host_f32(y)


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "qmm_*.npz"))), ids=os.path.basename)
def test_qmm_golden(path):
    g = load_golden(os.path.basename(path))
    y = _run(g["x"], g["w"], g["scales"], g["biases"])
    assert_close_rel(y, g["y"], REL, path)
    assert_close_rel(y, g["y"], REL_TIGHT, path)


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "qmm_*.npz"))), ids=os.path.basename)
def test_dequant_golden_bit_exact(path):
    import tsb

    g = load_golden(os.path.basename(path))
    out = tsb.dequantize(dev_u32(g["w"]), dev_bf16(g["scales"]), dev_bf16(g["biases"]))
    torch.cuda.synchronize()
    assert np.array_equal(host_bf16_bits(out), g["deq"])


def test_qmm_config1_seed0():
    """The small case: x [16, 5120] ~ N(0,1), W [6144, 5120] ~ N(0, 0.02), seed 0."""
    x, wq, s, b = gen.config1()
    y = _run(x, wq, s, b)
    ref = qmm.qmm(x, wq, s, b)
    assert_close_rel(y, ref, REL, "config1")
    assert_close_rel(y, ref, REL_TIGHT, "config1")


@pytest.mark.parametrize("m", [1, 2, 3, 4, 5, 8, 16, 31, 32, 33, 48, 64, 65, 128])
@pytest.mark.parametrize("nk", [(6144, 5120), (34816, 5120), (5120, 17408)])
def test_qmm_sweep_sampled_rows(m, nk):
    """The sweep shapes at every sweep M (plus odd M; 33-64 on 34816x5120 run the
    verify kernel's whole-tile configuration, the other shapes its default);
    the oracle is evaluated on a seeded sample of 384 output rows (all of K)."""
    import tsb

    n, k = nk
    rng = np.random.default_rng(1000 + m)
    # weights made on the device (fast), with the same quantizer as the oracle
    torch.manual_seed(1000 + m)
    wf = torch.randn(n, k, device="cuda") * 0.02
    wq, s, b = tsb.quantize(wf)
    x = gen.x_bf16(rng, m, k)
    y = tsb.quantized_matmul(dev_bf16(x), wq, s, b)
    torch.cuda.synchronize()
    rows = np.sort(rng.choice(n, size=384, replace=False))
    wq_h = wq[rows].cpu().numpy().view(np.uint32)
    ref = qmm.qmm(x, wq_h, host_bf16_bits(s[rows]), host_bf16_bits(b[rows]))
    got = host_f32(y)[:, rows]
    assert_close_rel(got, ref, REL, f"M={m} {nk}")
    assert_close_rel(got, ref, REL_TIGHT, f"M={m} {nk}")


def test_dequant_full_size_sampled_rows_bit_exact():
    import tsb

    n, k = 34816, 5120
    torch.manual_seed(5)
    wq, s, b = tsb.quantize(torch.randn(n, k, device="cuda") * 0.02)
    out = tsb.dequantize(wq, s, b)
    torch.cuda.synchronize()
    rows = np.random.default_rng(5).choice(n, size=256, replace=False)
    ref = qmm.dequantize(wq[rows].cpu().numpy().view(np.uint32), host_bf16_bits(s[rows]), host_bf16_bits(b[rows]))
    assert np.array_equal(host_bf16_bits(out[rows]), ref)


def test_qmm_ldy_writes_into_wider_buffer():
    """The N-shard contract: y rows of stride ldy > N, columns >= N untouched."""
    from tsb import ops

    g = load_golden("qmm_3.npz")  # M=16, N=128, K=640
    m, n = g["y"].shape
    ldy = 3 * n
    buf = torch.full((m, ldy), 7.0, dtype=torch.bfloat16, device="cuda")
    ops.quantized_matmul_into(dev_bf16(g["x"]), dev_u32(g["w"]), dev_bf16(g["scales"]), dev_bf16(g["biases"]),
                              buf[:, n:], ldy)
    torch.cuda.synchronize()
    h = host_f32(buf)
    assert np.all(h[:, :n] == 7.0) and np.all(h[:, 2 * n:] == 7.0)
    assert_close_rel(h[:, n:2 * n], g["y"], REL_TIGHT, "ldy")


def test_qmm_declines_and_rejects():
    import tsb

    x = torch.zeros(4, 128, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(96, 16, dtype=torch.int32, device="cuda")
    s = torch.zeros(96, 2, dtype=torch.bfloat16, device="cuda")
    assert tsb.quantized_matmul(x, w, s, s) is None  # N % 128: declined, caller falls back
    assert tsb.quantized_matmul(x, w, s, s, group_size=32) is None
    assert tsb.quantized_matmul(x.float(), w, s, s) is None


@pytest.mark.parametrize("m,n,k", [(256, 256, 128), (300, 128, 192), (513, 384, 640), (1024, 512, 1024),
                                   (257, 1024, 320)])
def test_qmm_gemm_path_full_oracle(m, n, k):
    """The tcgen05 GEMM path (M >= 256), odd M and N % 256 != 0 included."""
    rng = np.random.default_rng(7000 + m + n + k)
    x = gen.x_bf16(rng, m, k)
    wq, s, b = gen.weights_w4g64(rng, n, k)
    y = _run(x, wq, s, b)
    ref = qmm.qmm(x, wq, s, b)
    assert_close_rel(y, ref, REL, f"gemm {m}x{n}x{k}")
    assert_close_rel(y, ref, REL_TIGHT, f"gemm {m}x{n}x{k}")


@pytest.mark.parametrize("nk", [(34816, 5120), (5120, 17408), (6144, 5120)])
def test_qmm_prefill_config3_sampled(nk):
    """The prefill case: M = 4096; the oracle checks 48 x-rows x 256 weight rows."""
    import tsb

    n, k = nk
    m = 4096
    torch.manual_seed(3000 + n)
    wq, s, b = tsb.quantize(torch.randn(n, k, device="cuda") * 0.02)
    rng = np.random.default_rng(3000 + n)
    x = gen.x_bf16(rng, m, k)
    y = tsb.quantized_matmul(dev_bf16(x), wq, s, b)
    torch.cuda.synchronize()
    rows = np.sort(rng.choice(m, size=48, replace=False))
    cols = np.sort(rng.choice(n, size=256, replace=False))
    ref = qmm.qmm(x[rows], wq[cols].cpu().numpy().view(np.uint32), host_bf16_bits(s[cols]), host_bf16_bits(b[cols]))
    got = host_f32(y)[rows][:, cols]
    assert_close_rel(got, ref, REL, f"prefill {nk}")
    assert_close_rel(got, ref, REL_TIGHT, f"prefill {nk}")


@pytest.mark.parametrize("m,n,k", [(16, 6144, 5120), (1, 1024, 5120), (64, 384, 17408), (128, 128, 640)])
def test_qmm_split_tiles_and_workspace_left_clear(m, n, k):
    """Shapes whose row tiles are split across CTAs (stream-K parts joined through
    the workspace): full oracle check, twice in a row, and the workspace's
    completion flags are all zero again afterwards."""
    import tsb
    from tsb import _lib, ops

    rng = np.random.default_rng(9100 + m + n + k)
    x = gen.x_bf16(rng, m, k)
    wq, s, b = gen.weights_w4g64(rng, n, k)
    ref = qmm.qmm(x, wq, s, b)
    for _ in range(2):
        y = _run(x, wq, s, b)
        assert_close_rel(y, ref, REL_TIGHT, f"split {m}x{n}x{k}")
    lib = _lib.load()
    nbytes = lib.tsb_qmm_workspace_bytes(m, n, k)
    ws = ops.qmm_workspace(nbytes, "cuda")
    torch.cuda.synchronize()
    # flags are [tiles][maxp] uint32 words at the start of a fixed 64 KB flag
    # region (the kernel's plan for this device); partials follow it
    tiles, nst = n // 128, (k // 64 + 3) // 4
    units = tiles * nst
    ctas = max(1, min(torch.cuda.get_device_properties(0).multi_processor_count, units // 2))
    maxp = -(-nst // (units // ctas)) + 1
    flags = ws[: 64 * 1024].view(torch.int32).cpu().numpy()
    assert tiles * maxp <= flags.size
    assert not np.any(flags), "completion flags left set"


def test_qmm_workspace_too_small_refused():
    from tsb import _lib

    lib = _lib.load()
    x = torch.zeros(16, 5120, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(6144, 640, dtype=torch.int32, device="cuda")
    s = torch.zeros(6144, 80, dtype=torch.bfloat16, device="cuda")
    y = torch.empty(16, 6144, dtype=torch.bfloat16, device="cuda")
    small = torch.zeros(256, dtype=torch.uint8, device="cuda")
    st = lib.tsb_qmm_w4g64(x.data_ptr(), w.data_ptr(), s.data_ptr(), s.data_ptr(), y.data_ptr(), 16, 6144, 5120,
                           6144, small.data_ptr(), small.numel(), None)
    assert st == _lib.TSB_EWORKSPACE
    st = lib.tsb_qmm_w4g64(x.data_ptr(), w.data_ptr(), s.data_ptr(), s.data_ptr(), y.data_ptr(), 16, 6144, 5120,
                           6144, None, 0, None)
    assert st == _lib.TSB_EWORKSPACE


def test_device_status_clean_after_runs():
    """No bounded device-side wait has given up during the tests."""
    from tsb import _lib

    lib = _lib.load()
    assert lib.tsb_device_status(None, 0) == 0


@pytest.mark.parametrize("m", [1, 3, 16, 33, 64, 100])
@pytest.mark.parametrize("nk", [(256, 192), (384, 320), (128, 704), (640, 1088)])
def test_qmm_verify_odd_group_counts(m, nk):
    """K with a group count that is not a multiple of four (a partial last stage)
    or of eight (scales and biases read directly, not by TMA)."""
    n, k = nk
    rng = np.random.default_rng(4200 + m + n + k)
    x = gen.x_bf16(rng, m, k)
    wq, s, b = gen.weights_w4g64(rng, n, k)
    y = _run(x, wq, s, b)
    ref = qmm.qmm(x, wq, s, b)
    assert_close_rel(y, ref, REL_TIGHT, f"odd {m}x{n}x{k}")


def _bf16_round_once(v):
    """float64 -> bf16 value, one round-to-nearest-even from the exact value."""
    mant, ex = np.frexp(v)
    return np.ldexp(np.round(mant * 256) / 256, ex)


@pytest.mark.parametrize("m", [1, 2, 4, 16, 32, 64, 128, 256])
def test_effective_weights_rounding_rule(m):
    """The weight each matmul path multiplies with, read back through one-hot x
    rows (y[i] = W[:, k_i] exactly), for scale/bias pairs chosen so that q*s + b
    is not exact in float32: large |b| against a small s, scales on both sides of
    the kernels' 2^-5 fast-path limit, zero, subnormal and negative scales, and
    crafted cases (q = 6, s = 129 * 2^a, b = -1.5 * 2^(a-17)) whose float32
    rounding lands on a bf16 midpoint. The tcgen05 kernels (M > 2) dequantize
    with one bf16x2 fma, which rounds q*s + b once; tsb_dequant_w4g64 and the
    M <= 2 GEMV (group affine applied in float32 after integer dot products)
    round to float32 first, as the reference does (qmm_packed.py:200, 348,
    635). Both rules are pinned bit for bit, and they differ only on the
    crafted midpoint cases."""
    import tsb

    rng = np.random.default_rng(5)
    n, k = 256, 512
    g_n = k // 64
    codes = rng.integers(0, 16, size=(n, k)).astype(np.uint32)
    s = np.zeros((n, g_n))
    b = np.zeros((n, g_n))
    crafted = np.zeros((n, g_n), dtype=bool)
    for i in range(n):
        for g in range(g_n):
            f = i % 4
            if f == 0:
                s[i, g] = rng.uniform(0.002, 0.01)
                b[i, g] = -rng.uniform(0.02, 0.08)
            elif f == 1:
                s[i, g] = rng.uniform(1e-6, 1e-4) * rng.choice([-1, 1])
                b[i, g] = rng.uniform(1, 100) * rng.choice([-1, 1])
            elif f == 2:
                a = int(rng.integers(-20, -5))
                s[i, g] = 129 * 2.0 ** a
                b[i, g] = -1.5 * 2.0 ** (a - 17)
                codes[i, g * 64:(g + 1) * 64:2] = 6
                crafted[i, g] = True
            else:
                s[i, g] = [0.0, 1e-39, 0.5, -0.003, 3.0, -2e-5, 0.04, 2 ** -6][g % 8]
                b[i, g] = rng.uniform(-1, 1)
    s_bits = bf16.f32_to_bf16_bits(s.astype(np.float32))
    b_bits = bf16.f32_to_bf16_bits(b.astype(np.float32))
    sv = bf16.bf16_bits_to_f32(s_bits).astype(np.float64)
    bv = bf16.bf16_bits_to_f32(b_bits).astype(np.float64)
    exact = codes.reshape(n, g_n, 64) * sv[:, :, None] + bv[:, :, None]  # exact in float64
    once = _bf16_round_once(exact).reshape(n, k)
    twice = bf16.round_bf16(exact.astype(np.float32)).reshape(n, k).astype(np.float64)
    differ = once != twice
    assert differ.any() and np.all(np.repeat(crafted, 64, axis=1)[differ])
    wq = np.zeros((n, k // 8), dtype=np.uint32)
    for i in range(8):
        wq |= codes[:, i::8] << (4 * i)
    wd, sd, bd = dev_u32(wq), dev_bf16(s_bits), dev_bf16(b_bits)
    deq = bf16.bf16_bits_to_f32(host_bf16_bits(tsb.dequantize(wd, sd, bd))).astype(np.float64)
    assert np.array_equal(deq, twice)
    got = np.zeros((n, k))
    for k0 in range(0, k, m):
        x = torch.zeros(m, k, dtype=torch.bfloat16, device="cuda")
        idx = torch.arange(m, device="cuda")
        x[idx, (k0 + idx) % k] = 1
        y = host_f32(tsb.quantized_matmul(x, wd, sd, bd))
        for i in range(m):
            got[:, (k0 + i) % k] = y[i]
    want = twice if m <= 2 else once
    assert np.array_equal(got, want), int(np.sum(got != want))


@pytest.mark.parametrize("m,n,k", [(1100, 7680, 1024), (4096, 5120, 1536)])
def test_qmm_gemm_split_tail(m, n, k):
    """Prefill shapes whose tiles fill the SMs' last wave poorly: the last tiles
    are split along K (float parts in the workspace, added in a fixed order by
    a finishing kernel). Full oracle check twice, the second time over a
    workspace whose parts region holds garbage (the verify path leaves its
    partials there), bit-identical results, and the same result within
    tolerance when no workspace is given (every tile whole)."""
    import tsb
    from tsb import _lib, ops

    rng = np.random.default_rng(8800 + m + n + k)
    x = gen.x_bf16(rng, m, k)
    wq, s, b = gen.weights_w4g64(rng, n, k)
    lib = _lib.load()
    nbytes = lib.tsb_qmm_workspace_bytes(m, n, k)
    assert nbytes > 64 * 1024  # a split tail on this device (148 SMs)
    ref = qmm.qmm(x, wq, s, b)
    y = _run(x, wq, s, b)
    assert_close_rel(y, ref, REL_TIGHT, f"split tail {m}x{n}x{k}")
    ws = ops.qmm_workspace(nbytes, "cuda")
    ws[64 * 1024:nbytes].fill_(0x7F)  # float 3.4e38 in every word of the parts region
    y2 = _run(x, wq, s, b)
    ws[64 * 1024:nbytes].zero_()
    assert np.array_equal(y2, y), "split tail not deterministic"
    assert not torch.any(ws[:64 * 1024]).item(), "count region left non-zero"
    xd, wd, sd, bd = dev_bf16(x), dev_u32(wq), dev_bf16(s), dev_bf16(b)
    y0 = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    st = lib.tsb_qmm_w4g64(xd.data_ptr(), wd.data_ptr(), sd.data_ptr(), bd.data_ptr(), y0.data_ptr(), m, n, k, n,
                           None, 0, torch.cuda.current_stream().cuda_stream)
    assert st == 0
    assert_close_rel(host_f32(y0), ref, REL_TIGHT, "no workspace")
