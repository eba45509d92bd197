"""The reference-facing operators over torch CUDA tensors.

Each function mirrors the call the reference makes on its hot path, with the
same argument names and meaning:

  quantized_matmul(x, w, scales, biases, transpose=True, group_size=64, bits=4)
      = mx.quantized_matmul as called by the patched nn.QuantizedLinear
        (mlx-tree-spec src/mlx_tree_spec/packed_linear.py:83-104, :97)
  dequantize(w, scales, biases, group_size=64, bits=4)
      = mx.dequantize (tests/test_units.py:108), bit-exact rule
  ancestor_bits(parents)
      = tree_flash.ancestor_bits over Tree.anc (tree_flash.py:146-148,
        tree_verify.py:66-121)
  tree_flash(queries, cache, scale, bits, tail=None, stats=False)
      = tree_flash.tree_flash (tree_flash.py:151-196); also takes `parents=`
        so the mask is built inside the kernel.
  mask_bits(mask, tail)
      = the inverse of Tree.mask (tree_verify.py:131-139): an SDPA mask -> bits
  sdpa(queries, keys, values, cache, scale, mask, fallback=None)
      = the mlx-lm SDPA hook of long_attention.install (long_attention.py:
        69-88) with kv8.attention's routing (kv8.py:162-188)
  keep_kv(cache, off0, nodes) / commit(caches, off0, nodes)
      = tree_verify._keep_kv / the attention-cache part of tree_verify.commit
        (tree_verify.py:487-516): keep the accepted path's K/V rows.

Decline behaviour follows the reference: an unsupported shape or format
returns None (the caller falls back), contract violations raise. All work is
enqueued on torch's current CUDA stream; scratch memory comes from a per-device
workspace owned here (the C ABI itself never allocates).
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import (TSB_EUNSUPPORTED, TSB_KV_BF16, TSB_KV_MLX_Q8_G64, TSB_KV_REF_Q8_ROW, TSB_MASK_BF16,
                   TSB_MASK_BOOL, TSB_MASK_F16, TSB_MASK_F32, check)

_WS: dict[int, torch.Tensor] = {}


def workspace(nbytes: int, device) -> torch.Tensor:
    """A per-device uint8 scratch buffer of at least nbytes (grown, never shrunk)."""
    dev = torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    buf = _WS.get(idx)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=torch.device("cuda", idx))
        _WS[idx] = buf
    return buf


_QWS: dict[int, torch.Tensor] = {}


def qmm_workspace(nbytes: int, device) -> torch.Tensor:
    """The per-device workspace of the verify qmm: zero-initialised, used for nothing else.

    It holds completion flags the kernel leaves zero after every call, so it is
    allocated with zeros once (and again, zeroed, when it has to grow) and never
    shared with the attention scratch."""
    dev = torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    buf = _QWS.get(idx)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=torch.device("cuda", idx))
        _QWS[idx] = buf
    return buf


# The raw current-stream handle: torch's own C++ accessor when this build of
# torch has it (a fraction of the ~2 us that torch.cuda.current_stream() costs
# per call, which matters for M = 1 calls of a few microseconds), else the
# public API.
_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(t: torch.Tensor) -> int:
    if _RAW_STREAM is not None:
        return _RAW_STREAM(t.device.index)
    return torch.cuda.current_stream(t.device).cuda_stream


_QWS_BYTES: dict[tuple, int] = {}


def _qmm_ws_bytes(lib, m: int, n: int, k: int, dev: int) -> int:
    """tsb_qmm_workspace_bytes, remembered per (M, N, K, device) on the host side."""
    key = (m, n, k, dev)
    v = _QWS_BYTES.get(key)
    if v is None:
        v = _QWS_BYTES[key] = lib.tsb_qmm_workspace_bytes(m, n, k)
    return v


def _ptr(t):
    return None if t is None else t.data_ptr()


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("tsb operators take CUDA tensors (there is no CPU path)")


def quantized_matmul(x, w, scales, biases, transpose: bool = True, group_size: int = 64, bits: int = 4,
                     out: torch.Tensor | None = None):
    """y = x @ dequantize(w, scales, biases).T for x (..., K) bf16.

    w: uint32 (N, K/8) [torch.int32 or torch.uint32 storage]; scales, biases:
    bf16 (N, K/64). Returns (..., N) bf16, or None when declined (the shape
    or configuration is not one this kernel takes)."""
    _require_cuda(x, w, scales, biases)
    if not transpose or group_size != 64 or bits != 4:
        return None
    if x.dtype != torch.bfloat16 or scales.dtype != torch.bfloat16 or biases.dtype != torch.bfloat16:
        return None
    k = x.shape[-1]
    n = w.shape[0]
    if w.shape[-1] * 8 != k or scales.shape != (n, k // 64) or biases.shape != (n, k // 64):
        raise ValueError(f"inconsistent shapes: x {tuple(x.shape)}, w {tuple(w.shape)}, scales {tuple(scales.shape)}")
    x2 = x.reshape(-1, k)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    m = x2.shape[0]
    if out is None:
        out = torch.empty((*x.shape[:-1], n), dtype=torch.bfloat16, device=x.device)
    lib = _lib.load()
    ws = qmm_workspace(_qmm_ws_bytes(lib, m, n, k, x.device.index), x.device)
    st = lib.tsb_qmm_w4g64(_ptr(x2), _ptr(w), _ptr(scales), _ptr(biases), _ptr(out), m, n, k, n,
                           _ptr(ws), ws.numel(), _stream(x))
    if check(st, "tsb_qmm_w4g64") == TSB_EUNSUPPORTED:
        return None
    return out


def quantized_matmul_into(x2, w, scales, biases, y, ldy: int):
    """Low-level: x2 (M, K) contiguous -> y (an (M, ldy) buffer, N columns written).

    Used by the N-sharded path to write a shard straight into a wider buffer."""
    m, k = x2.shape
    n = w.shape[0]
    lib = _lib.load()
    ws = qmm_workspace(_qmm_ws_bytes(lib, m, n, k, x2.device.index), x2.device)
    st = lib.tsb_qmm_w4g64(_ptr(x2), _ptr(w), _ptr(scales), _ptr(biases), _ptr(y), m, n, k, ldy,
                           _ptr(ws), ws.numel(), _stream(x2))
    return check(st, "tsb_qmm_w4g64")


def dequantize(w, scales, biases, group_size: int = 64, bits: int = 4):
    """Bit-exact dequantization: bf16 (N, K) = bf16_rne(fmaf(q, s, b))."""
    _require_cuda(w, scales, biases)
    if group_size != 64 or bits != 4:
        return None
    n = w.shape[0]
    k = w.shape[1] * 8
    out = torch.empty((n, k), dtype=torch.bfloat16, device=w.device)
    lib = _lib.load()
    st = lib.tsb_dequant_w4g64(_ptr(w), _ptr(scales), _ptr(biases), _ptr(out), n, k, _stream(w))
    if check(st, "tsb_dequant_w4g64") == TSB_EUNSUPPORTED:
        return None
    return out


def ancestor_bits(parents, depth: bool = False):
    """parents int32 (T,) or (B, T) on the GPU -> uint64 masks (as int64 storage),
    and the node depths if asked."""
    _require_cuda(parents)
    p = parents.to(torch.int32)
    squeeze = p.dim() == 1
    p2 = p.reshape(1, -1) if squeeze else p
    p2 = p2.contiguous()
    b, t = p2.shape
    bits = torch.empty((b, t), dtype=torch.int64, device=p.device)
    dep = torch.empty((b, t), dtype=torch.int32, device=p.device) if depth else None
    lib = _lib.load()
    st = lib.tsb_tree_ancestor_bits(_ptr(p2), b, t, _ptr(bits), _ptr(dep), _stream(p2))
    if check(st, "tsb_tree_ancestor_bits") == TSB_EUNSUPPORTED:
        return None
    if squeeze:
        bits = bits[0]
        dep = dep[0] if dep is not None else None
    return (bits, dep) if depth else bits


_MASK_TYPES = {torch.bool: TSB_MASK_BOOL, torch.uint8: TSB_MASK_BOOL, torch.bfloat16: TSB_MASK_BF16,
               torch.float16: TSB_MASK_F16, torch.float32: TSB_MASK_F32}


def mask_bits(mask, tail: int):
    """An SDPA mask on the GPU -> (bits, bad): the inverse of Tree.mask
    (tree_verify.py:131-139). mask (..., L): boolean (True visible) or additive
    (0 visible, -inf hidden) in bf16 / fp16 / float32. bits int64 (...,): bit
    j set iff column L - tail + j is visible. bad: int32 (1,) on the device,
    the number of rows the bit form cannot express (a hidden column before the
    last `tail`, or an additive value other than 0 and -inf); read it before
    trusting bits. None if the mask type or tail (> 64) is not taken."""
    _require_cuda(mask)
    dt = _MASK_TYPES.get(mask.dtype)
    if dt is None or mask.dim() < 1 or not 0 <= tail <= min(64, mask.shape[-1]):
        return None
    L = mask.shape[-1]
    lead = tuple(mask.shape[:-1])
    m2 = mask.reshape(-1, L)
    if m2.stride(-1) != 1 or (m2.shape[0] > 1 and m2.stride(0) < L):
        m2 = m2.contiguous()
    rows = m2.shape[0]
    row_stride = m2.stride(0) if rows > 1 else L
    bits = torch.empty(rows, dtype=torch.int64, device=mask.device)
    bad = torch.empty(1, dtype=torch.int32, device=mask.device)
    lib = _lib.load()
    st = lib.tsb_tree_mask_bits(_ptr(m2), dt, rows, L, row_stride, tail, _ptr(bits), _ptr(bad), _stream(m2))
    if check(st, "tsb_tree_mask_bits") == TSB_EUNSUPPORTED:
        return None
    return bits.reshape(lead), bad


def _kv_planes(cache):
    """(format, k, k_scales, k_biases, v, v_scales, v_biases) of a cache object."""
    fmt = getattr(cache, "kv_format", None)
    if fmt is None:
        fmt = TSB_KV_REF_Q8_ROW if getattr(cache, "k_scale", None) is not None else TSB_KV_BF16
    if fmt == TSB_KV_BF16:
        return fmt, cache.keys, None, None, cache.values, None, None
    if fmt == TSB_KV_REF_Q8_ROW:
        return fmt, cache.keys, cache.k_scale, None, cache.values, cache.v_scale, None
    if fmt == TSB_KV_MLX_Q8_G64:
        return fmt, cache.keys, cache.k_scales, cache.k_biases, cache.values, cache.v_scales, cache.v_biases
    raise ValueError(f"unknown kv format {fmt}")


def tree_flash(queries, cache, scale: float, bits=None, tail: int | None = None, stats: bool = False,
               parents=None, out=None):
    """Tree-mask attention of `queries` (B, Hq, n, D) over `cache`.

    cache: any object with keys/values (B, Hkv, capacity, ...) and `offset`
    (valid rows, the nodes' own rows last), optionally k_scale/v_scale (the
    reference's int8-row format) or kv_format = TSB_KV_MLX_Q8_G64 with
    k_scales/k_biases/v_scales/v_biases. Visibility per the reference: node q
    sees the rows before the last `tail` (default n) plus the tail rows set in
    bits[q] (uint64 masks as int64, shape (n,) or (B, n); tail 0 = all rows).
    With parents= (int32 (n,) or (B, n)) the masks are built in the kernel.

    Returns out (B, Hq, n, D) bf16, or (out, maxs, sums) with stats=True where
    maxs = log-sum-exp of each row's visible scores and sums = 1 (a single
    block: merge with more keys as tree_verify.py:389-401 does), or None when
    declined. `out` (optional): a (B, Hq, n, D) bf16 buffer to write into."""
    fmt, k, ks, kb, v, vs, vb = _kv_planes(cache)
    _require_cuda(queries, k, v)
    if queries.dtype != torch.bfloat16:
        return None
    bsz, hq, n, d = queries.shape
    hkv, cap = k.shape[1], k.shape[2]
    n_kv = int(cache.offset)
    if parents is not None:
        p = parents.to(device=queries.device, dtype=torch.int32)
        p = p.reshape(1, n).expand(bsz, n) if p.dim() == 1 else p
        p = p.contiguous()
        bits_t = None
        tail_v = n
    else:
        if bits is None:
            return None
        bt = bits if isinstance(bits, torch.Tensor) else torch.tensor([int(b) if int(b) < 2**63 else int(b) - 2**64 for b in bits], dtype=torch.int64)
        bt = bt.to(device=queries.device, dtype=torch.int64)
        bt = bt.reshape(1, n).expand(bsz, n) if bt.dim() == 1 else bt
        bits_t = bt.contiguous()
        p = None
        tail_v = n if tail is None else int(tail)
    q = queries.contiguous()
    out = torch.empty_like(q) if out is None else out
    lse = torch.empty((bsz, hq, n), dtype=torch.float32, device=q.device) if stats else None
    lib = _lib.load()
    ws = workspace(lib.tsb_tree_attn_workspace_bytes(bsz, n, hq, hkv, d, n_kv, fmt), q.device)
    st = lib.tsb_tree_attn(_ptr(q), _ptr(k), _ptr(ks), _ptr(kb), _ptr(v), _ptr(vs), _ptr(vb), fmt,
                           _ptr(p), _ptr(bits_t), bsz, n, hq, hkv, d, n_kv, tail_v, cap, float(scale),
                           _ptr(out), _ptr(lse), _ptr(ws), ws.numel(), _stream(q))
    if check(st, "tsb_tree_attn") == TSB_EUNSUPPORTED:
        return None
    if stats:
        return out, lse[..., None], torch.ones_like(lse)[..., None]
    return out


class _Rows:
    """Keys and values with no cache object around them: every row is a key."""

    def __init__(self, keys, values):
        self.keys, self.values, self.offset = keys, values, keys.shape[2]


def _causal_bits(n: int, device) -> torch.Tensor:
    """Tail-causal masks: node q sees tail rows 0..q (kv8.py:194-197 causal_bits)."""
    return torch.tensor([(1 << (q + 1)) - 1 if q < 63 else -1 for q in range(n)], dtype=torch.int64, device=device)


def _sdpa_tree(queries, keys, values, cache, scale, mask):
    n = queries.shape[2]
    if n > 64:
        return None
    src = cache if cache is not None and getattr(cache, "keys", None) is not None else _Rows(keys, values)
    if mask is None or (isinstance(mask, str) and mask == "causal"):
        bits = _causal_bits(n, queries.device)
    elif not isinstance(mask, torch.Tensor):
        return None
    else:
        m = mask
        if m.dim() < 2 or m.shape[-2] != n or m.shape[-1] != int(src.offset):
            return None
        if m.dim() == 4:  # (B, heads, n, L): one mask for every head only
            if m.shape[1] != 1:
                return None
            m = m[:, 0]
        if m.dim() == 3:  # (B, n, L)
            if m.shape[0] == 1:
                m = m[0]
            elif m.shape[0] != queries.shape[0]:
                return None
        if m.dim() not in (2, 3):
            return None
        r = mask_bits(m, n)
        if r is None:
            return None
        bits, bad = r
        if int(bad.item()) != 0:
            return None
    return tree_flash(queries, src, scale, bits, tail=n)


def sdpa(queries, keys, values, cache, scale, mask, *args, fallback=None, **kwargs):
    """The mlx-lm scaled_dot_product_attention hook (long_attention.py:69-88,
    install().sdpa) over tsb's tree attention, with kv8.attention's routing of
    the 8-bit caches (kv8.py:162-188) and batch_attention's SDPA fallback
    (tree_verify.py:359-366).

    queries (B, Hq, n, D) bf16. cache: a KVCache / Q8KVCache / MLXQ8KVCache
    whose first `offset` rows are the keys, the queries' own rows last; with
    cache None, keys and values (B, Hkv, L, D) bf16 are all keys. mask: None
    or "causal" (the reference's tail-causal rule on this path: query i sees
    the rows before the last n and tail rows 0..i), or a boolean / additive
    (0 or -inf) tensor whose last two dims are (n, keys) and whose leading
    dims are 1 or the batch over requests and 1 over heads, such as
    Tree.mask (tree_verify.py:131-139). A tensor mask is converted by
    tsb_tree_mask_bits, which costs one device->host read of its status.

    Returns out (B, Hq, n, D) bf16. What the kernel does not take (a mask that
    is not a visibility mask, n > 64, extra arguments, a shape the kernel
    declines) goes to fallback(queries, keys, values, cache=cache,
    scale=scale, mask=mask, *args, **kwargs) -- the hooked original, as the
    reference's hook does -- or returns None with no fallback."""
    out = None if args or kwargs else _sdpa_tree(queries, keys, values, cache, scale, mask)
    if out is None and fallback is not None:
        return fallback(queries, keys, values, *args, cache=cache, scale=scale, mask=mask, **kwargs)
    return out


def _commit_plan(bsz: int, off0, nodes):
    """(per_request, offsets, paths, new offsets) of a commit over bsz requests."""
    per_request = not isinstance(off0, int)
    offs = [int(o) for o in off0] if per_request else [int(off0)] * bsz
    paths = [[int(i) for i in p] for p in nodes] if per_request else [[int(i) for i in nodes]] * bsz
    if len(offs) != bsz or len(paths) != bsz:
        raise ValueError(f"keep_kv: {len(offs)} offsets and {len(paths)} paths for {bsz} requests")
    return per_request, offs, paths, [o + len(p) for o, p in zip(offs, paths)]


def _commit_launch(caches, offs, paths):
    """One tsb_kv_commit_layers launch over caches of one format and shape."""
    planes = [_kv_planes(c) for c in caches]
    fmt = planes[0][0]
    k0 = planes[0][1]
    for pl in planes:
        _require_cuda(pl[1], pl[4])
        if not all(t is None or t.is_contiguous() for t in pl[1:]):
            raise ValueError("keep_kv: cache tensors must be contiguous")
        if pl[0] != fmt or pl[1].shape != k0.shape or pl[1].dtype != k0.dtype or pl[1].device != k0.device:
            raise ValueError("commit: every cache of one launch must share format, shape and device")
    bsz, hkv, cap = k0.shape[0], k0.shape[1], k0.shape[2]
    d = (k0.shape[3] * 4) if fmt == TSB_KV_MLX_Q8_G64 else k0.shape[3]
    max_keep = max(1, max(len(p) for p in paths))
    flat = [0] * (bsz * max_keep)
    for b, p in enumerate(paths):
        flat[b * max_keep:b * max_keep + len(p)] = p
    i32, vp = ctypes.c_int32, ctypes.c_void_p
    n = len(planes)
    arrays = [(vp * n)(*[_ptr(pl[j]) for pl in planes]) if planes[0][j] is not None else None for j in range(1, 7)]
    lib = _lib.load()
    st = lib.tsb_kv_commit_layers(fmt, n, arrays[0], arrays[1], arrays[2], arrays[3], arrays[4], arrays[5], bsz, hkv,
                                  d, cap, (i32 * bsz)(*offs), (i32 * len(flat))(*flat),
                                  (i32 * bsz)(*[len(p) for p in paths]), max_keep, _stream(k0))
    if check(st, "tsb_kv_commit_layers") == TSB_EUNSUPPORTED:
        raise ValueError(f"keep_kv: unsupported cache (D={d}, B={bsz}, path length {max_keep}, {n} layers)")


def keep_kv(cache, off0, nodes):
    """Keep only the accepted path of a finished tree pass in `cache`
    (mlx-tree-spec src/mlx_tree_spec/tree_verify.py:487-496 _keep_kv; the int8
    cache's take_rows, kv8.py:143-148): rows off0 + nodes[i] move to rows
    off0 + i of every KV head's keys and values (and scales / biases).

    off0 int with nodes a list of ints: the reference's form, the same path for
    every request of the cache; cache.offset becomes off0 + len(nodes) and that
    is returned. off0 a sequence with nodes a list of lists: one tree region
    start and path per request; the new per-request offsets are returned (the
    caller holds them) and cache.offset is left alone. A path equal to
    range(len(path)) for every request moves nothing and launches nothing, as
    the reference skips its take for a contiguous path."""
    return commit([cache], off0, nodes)[0]


_MAX_LAYERS_PER_LAUNCH = 48


def commit(caches, off0, nodes):
    """keep_kv over every layer's cache (tree_verify.py:499-516 commit, its
    attention-cache part: the KVCache layers and the MTP caches), as one
    launch per 48 caches of the same format and shape. Returns each cache's
    keep_kv result."""
    caches = list(caches)
    if not caches:
        return []
    k0 = _kv_planes(caches[0])[1]
    per_request, offs, paths, new_offs = _commit_plan(k0.shape[0], off0, nodes)
    if any(p != list(range(len(p))) for p in paths):
        groups: dict = {}
        for c in caches:
            fmt, k = _kv_planes(c)[:2]
            groups.setdefault((fmt, tuple(k.shape), k.dtype, str(k.device)), []).append(c)
        for group in groups.values():
            if group[0] is not caches[0] and _kv_planes(group[0])[1].shape[0] != k0.shape[0]:
                raise ValueError("commit: every cache must hold the same requests")
            for i in range(0, len(group), _MAX_LAYERS_PER_LAUNCH):
                _commit_launch(group[i:i + _MAX_LAYERS_PER_LAUNCH], offs, paths)
    if per_request:
        return [list(new_offs) for _ in caches]
    for c in caches:
        c.offset = new_offs[0]
    return [new_offs[0]] * len(caches)
