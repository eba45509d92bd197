"""ctypes binding of libtsb.so (the C ABI declared in include/tsb.h).

The library is built in-tree (tsb/libtsb.so) by tsb.build. There is no
fallback: if the shared object is missing or does not load, importing the ops
raises, so a GPU run can never silently compute on the CPU.
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libtsb.so")

TSB_OK = 0
TSB_EUNSUPPORTED = 1
TSB_EINVAL = 2
TSB_ECUDA = 3
TSB_ETIMEOUT = 4
TSB_EWORKSPACE = 5

TSB_KV_BF16 = 0
TSB_KV_MLX_Q8_G64 = 1
TSB_KV_REF_Q8_ROW = 2

TSB_MASK_BOOL = 0
TSB_MASK_BF16 = 1
TSB_MASK_F16 = 2
TSB_MASK_F32 = 3

TSB_MAX_GATHER_RANKS = 8


class GatherT(ctypes.Structure):
    """tsb_gather_t: each rank's output buffer and signal block, as mapped here."""

    _fields_ = [("world", ctypes.c_int), ("rank", ctypes.c_int),
                ("y", ctypes.c_void_p * TSB_MAX_GATHER_RANKS),
                ("sig", ctypes.c_void_p * TSB_MAX_GATHER_RANKS)]


# Every symbol include/tsb.h declares, with (restype, argtypes).
_P, _I, _Z, _F, _LL = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.c_float, ctypes.c_longlong
SIGNATURES = {
    "tsb_strerror": (ctypes.c_char_p, [_I]),
    "tsb_version": (_I, []),
    "tsb_device_status": (_I, [_P, _I]),
    "tsb_qmm_workspace_bytes": (_Z, [_I, _I, _I]),
    "tsb_qmm_w4g64": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P, _Z, _P]),
    "tsb_qmm_w4g64_gather": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, ctypes.POINTER(GatherT), _P, _Z, _P]),
    "tsb_dequant_w4g64": (_I, [_P, _P, _P, _P, _I, _I, _P]),
    "tsb_tree_ancestor_bits": (_I, [_P, _I, _I, _P, _P, _P]),
    "tsb_tree_mask_bits": (_I, [_P, _I, _I, _LL, _LL, _I, _P, _P, _P]),
    "tsb_tree_attn_workspace_bytes": (_Z, [_I, _I, _I, _I, _I, _I, _I]),
    "tsb_tree_attn": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _F,
                           _P, _P, _P, _Z, _P]),
    "tsb_add_rms_norm": (_I, [_P, _P, _P, _P, _P, _I, _I, _F, _P]),
    "tsb_qkv_prep": (_I, [_P, _I, _I, _I, _I, _I, _I, _P, _P, _F, _P, _I, _F, _F, _P, _I, _P, _P, _P, _P, _P, _P,
                          _I, _P, _P]),
    "tsb_attn_gate": (_I, [_P, _P, _I, _P, _I, _I, _I, _I, _P]),
    "tsb_swiglu": (_I, [_P, _P, _I, _I, _P]),
    "tsb_tree_attn_noalloc": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _F,
                                   _P, _P, _P]),
    "tsb_kv_commit": (_I, [_I, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _I, _P]),
    "tsb_kv_commit_layers": (_I, [_I, _I, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _I, _P]),
    "tsb_gdn_prep": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "tsb_tree_gated_delta": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P, _P]),
    "tsb_gdn_commit": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _P, _P]),
}


class TSBError(RuntimeError):
    def __init__(self, status: int, where: str):
        self.status = status
        super().__init__(f"{where}: {strerror(status)} (status {status})")


_lib = None


def load(path: str | None = None) -> ctypes.CDLL:
    """Load libtsb.so once and declare every exported signature."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise ImportError(f"libtsb.so not built: {p} is missing (run __graft_entry__.build() or python -m tsb.build)")
    lib = ctypes.CDLL(p)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def strerror(status: int) -> str:
    try:
        return load().tsb_strerror(status).decode()
    except ImportError:
        return f"status {status}"


def check(status: int, where: str) -> int:
    """Raise TSBError unless status is OK or a decline (returned to the caller)."""
    if status not in (TSB_OK, TSB_EUNSUPPORTED):
        raise TSBError(status, where)
    return status
