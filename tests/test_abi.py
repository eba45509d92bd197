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
