"""The C ABI: libtsb.so builds for sm_100a, loads, and exports every symbol
include/tsb.h declares. Host-only checks; nothing here launches a kernel."""

import ctypes
import os
import re

from conftest import ROOT


def header_symbols():
    src = open(os.path.join(ROOT, "include", "tsb.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(tsb_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol(lib_built):
    lib = ctypes.CDLL(lib_built)
    syms = header_symbols()
    assert "tsb_qmm_w4g64" in syms and "tsb_tree_attn" in syms
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in include/tsb.h but not exported"


def test_binding_covers_header(lib_built):
    from tsb import _lib

    assert set(header_symbols()) == set(_lib.SIGNATURES)
    lib = _lib.load()
    assert lib.tsb_version() >= 0x000100


def test_strerror_and_codes(lib_built):
    from tsb import _lib

    lib = _lib.load()
    for code in range(6):
        assert lib.tsb_strerror(code)
    assert b"unsupported" in lib.tsb_strerror(_lib.TSB_EUNSUPPORTED)
    assert lib.tsb_strerror(99) == b"unknown status"


def test_argument_checks_before_any_launch(lib_built):
    """Contract violations and declines return before touching the device."""
    from tsb import _lib

    lib = _lib.load()
    fake = 0x1000  # never dereferenced: every call below fails its host-side checks
    assert lib.tsb_qmm_w4g64(None, fake, fake, fake, fake, 1, 128, 64, 128, fake, 1 << 20, None) == _lib.TSB_EINVAL
    assert lib.tsb_qmm_w4g64(fake, fake, fake, fake, fake, 1, 100, 64, 128, fake, 1 << 20, None) == _lib.TSB_EUNSUPPORTED
    assert lib.tsb_qmm_w4g64(fake, fake, fake, fake, fake, 1, 128, 96, 128, fake, 1 << 20, None) == _lib.TSB_EUNSUPPORTED
    assert lib.tsb_qmm_w4g64(fake, fake, fake, fake, fake, 1, 128, 64, 64, fake, 1 << 20, None) == _lib.TSB_EINVAL
    assert lib.tsb_dequant_w4g64(fake, fake, fake, fake, 128, 100, None) == _lib.TSB_EINVAL
    assert lib.tsb_tree_ancestor_bits(fake, 1, 65, fake, None, None) == _lib.TSB_EUNSUPPORTED
    assert lib.tsb_tree_ancestor_bits(None, 1, 4, fake, None, None) == _lib.TSB_EINVAL
    args = dict(B=1, T=4, Hq=8, Hkv=2, D=256, n_kv=100, tail=4, cap=128)

    def attn(**kw):
        a = {**args, **kw}
        return lib.tsb_tree_attn(fake, fake, None, None, fake, None, None, kw.get("fmt", 0), fake, None,
                                 a["B"], a["T"], a["Hq"], a["Hkv"], a["D"], a["n_kv"], a["tail"], a["cap"],
                                 0.0625, fake, None, fake, 1 << 30, None)

    assert attn(D=128) == _lib.TSB_EUNSUPPORTED
    assert attn(Hq=6, Hkv=4) == _lib.TSB_EUNSUPPORTED
    assert attn(T=65) == _lib.TSB_EUNSUPPORTED
    assert attn(cap=50) == _lib.TSB_EINVAL
    assert attn(fmt=1) == _lib.TSB_EINVAL  # q8 g64 without scales/biases
    assert attn(fmt=7) == _lib.TSB_EUNSUPPORTED


def test_workspace_sizes_are_host_computable(lib_built):
    from tsb import _lib

    lib = _lib.load()
    # verify path: completion flags + partials of the row tiles split across CTAs
    assert lib.tsb_qmm_workspace_bytes(16, 6144, 5120) > 0
    assert lib.tsb_qmm_workspace_bytes(4096, 6144, 5120) == 0  # the prefill GEMM needs none
    assert lib.tsb_tree_attn_workspace_bytes(1, 32, 24, 4, 256, 32800, 0) > 0


def test_gather_and_decoder_checks_before_any_launch(lib_built):
    """The in-kernel-gather qmm and the decoder kernels refuse bad arguments on
    the host (nothing is launched: the pointers below are never dereferenced)."""
    import ctypes

    from tsb import _lib

    lib = _lib.load()
    fake = 0x1000
    g = _lib.GatherT()
    g.world, g.rank = 2, 0
    for p in range(2):
        g.y[p], g.sig[p] = fake, fake

    def gather(m=16, ns=1024, k=5120, ldy=2048, gg=g, x=fake):
        return lib.tsb_qmm_w4g64_gather(x, fake, fake, fake, m, ns, k, ldy, ctypes.byref(gg) if gg else None,
                                        fake, 1 << 20, None)

    assert gather(x=None) == _lib.TSB_EINVAL
    assert gather(gg=None) == _lib.TSB_EINVAL
    assert gather(ns=1000) == _lib.TSB_EUNSUPPORTED  # shard rows not a multiple of 128
    assert gather(ldy=1024) == _lib.TSB_EINVAL       # narrower than world * Ns
    assert gather(m=4096, ldy=1024) == _lib.TSB_EINVAL  # the prefill form checks the same
    bad = _lib.GatherT()
    bad.world, bad.rank = 2, 2
    assert gather(gg=bad) == _lib.TSB_EINVAL         # rank out of range
    bad.world, bad.rank = 9, 0
    assert gather(gg=bad) == _lib.TSB_EINVAL         # more ranks than TSB_MAX_GATHER_RANKS
    half = _lib.GatherT()
    half.world, half.rank = 2, 1
    half.y[0], half.sig[0] = fake, fake              # rank 1's buffers missing
    assert gather(gg=half) == _lib.TSB_EINVAL

    assert lib.tsb_add_rms_norm(fake, None, fake, None, fake, 4, 5121, 1e-6, None) == _lib.TSB_EUNSUPPORTED
    assert lib.tsb_add_rms_norm(None, None, fake, None, fake, 4, 5120, 1e-6, None) == _lib.TSB_EINVAL
    assert lib.tsb_add_rms_norm(fake, None, fake, None, fake, 4, 16392, 1e-6, None) == _lib.TSB_EUNSUPPORTED

    def prep(**kw):
        a = dict(ld=14336, B=4, T=32, Hq=24, Hkv=4, D=256, rope=64, base=1e7, fmt=0, cap=8224)
        a.update(kw)
        return lib.tsb_qkv_prep(fake, a["ld"], a["B"], a["T"], a["Hq"], a["Hkv"], a["D"], fake, fake, 1e-6, fake,
                                a["rope"], a["base"], 1.0, fake, a["fmt"], fake, None, None, fake, None, None,
                                a["cap"], fake, None)

    assert prep(D=128) == _lib.TSB_EUNSUPPORTED
    assert prep(rope=72) == _lib.TSB_EUNSUPPORTED   # rope dims must be a multiple of 16
    assert prep(ld=14000) == _lib.TSB_EINVAL         # narrower than the q/gate/k/v columns
    assert prep(fmt=1) == _lib.TSB_EINVAL            # MLX 8-bit without scales/biases
    assert prep(fmt=5) == _lib.TSB_EUNSUPPORTED
    assert prep(base=0.0) == _lib.TSB_EINVAL
    assert lib.tsb_attn_gate(fake, fake, 1000, fake, 4, 32, 24, 256, None) == _lib.TSB_EINVAL
    assert lib.tsb_swiglu(fake, fake, 128, 17404, None) == _lib.TSB_EUNSUPPORTED

    def keep(offs=(8, 8), paths=((0, 2, 3), (0, 1)), **kw):
        a = dict(fmt=0, B=2, Hkv=4, D=256, cap=96, max_keep=3)
        a.update(kw)
        i32 = ctypes.c_int32
        flat = [0] * (a["B"] * a["max_keep"])
        for b, p in enumerate(paths[:a["B"]]):
            flat[b * a["max_keep"]:b * a["max_keep"] + len(p)] = p
        n = [len(p) for p in paths[:a["B"]]]
        return lib.tsb_kv_commit(a["fmt"], fake, fake, fake, fake, fake, fake, a["B"], a["Hkv"], a["D"], a["cap"],
                                 (i32 * a["B"])(*offs[:a["B"]]), (i32 * len(flat))(*flat), (i32 * a["B"])(*n),
                                 a["max_keep"], None)

    # host-side contract checks of the tree commit (no launch reaches the GPU)
    assert keep(D=128) == _lib.TSB_EUNSUPPORTED
    assert keep(B=9, offs=(0,) * 9, paths=((0,),) * 9) == _lib.TSB_EUNSUPPORTED  # more than 8 requests
    assert keep(max_keep=65) == _lib.TSB_EUNSUPPORTED                             # path longer than 64
    assert keep(fmt=3) == _lib.TSB_EUNSUPPORTED
    assert keep(paths=((0, 2, 64), (0, 1))) == _lib.TSB_EINVAL                    # node past the tree width
    assert keep(paths=((0, 2, -1), (0, 1))) == _lib.TSB_EINVAL
    assert keep(offs=(8, 95)) == _lib.TSB_EINVAL                                  # destination past capacity
    assert keep(paths=((0, 1, 2, 3), (0,)), max_keep=3) == _lib.TSB_EINVAL         # n_keep > max_keep
    assert lib.tsb_kv_commit(0, None, None, None, fake, None, None, 1, 4, 256, 96, (ctypes.c_int32 * 1)(0),
                             (ctypes.c_int32 * 1)(0), (ctypes.c_int32 * 1)(1), 1, None) == _lib.TSB_EINVAL

    def layers(n, k=fake, v=fake):
        vp, i32 = ctypes.c_void_p, ctypes.c_int32
        ks = (vp * n)(*[k] * n)
        vs = (vp * n)(*([v] * (n - 1) + [None]))   # the last layer's V pointer missing
        return lib.tsb_kv_commit_layers(0, n, ks, None, None, vs, None, None, 1, 4, 256, 96, (i32 * 1)(0),
                                        (i32 * 2)(0, 2), (i32 * 1)(2), 2, None)

    assert layers(49) == _lib.TSB_EUNSUPPORTED      # more than 48 layers per launch
    assert layers(3) == _lib.TSB_EINVAL             # a null plane in layer 2
    assert lib.tsb_kv_commit_layers(0, 0, None, None, None, None, None, None, 1, 4, 256, 96, None, None, None, 1,
                                    None) == _lib.TSB_EINVAL
