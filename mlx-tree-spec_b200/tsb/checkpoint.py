"""MLX checkpoint loader: safetensors QuantizedLinear weights -> device buffers.

The reference loads an mlx-lm checkpoint (safetensors shards + config.json)
and repacks every eligible 4-bit QuantizedLinear for its kernels
(mlx-tree-spec src/mlx_tree_spec/packed_linear.py:136-156 install, eligibility
at packed_linear.py:49-58, the repack itself pack_nax at qmm_packed.py:223-232).
The kernels here read MLX's own layout (uint32 words of eight 4-bit codes, bf16
scales and biases per 64 values), so loading is a byte copy with no repack:

  * safetensors is parsed here (8-byte little-endian header length, JSON
    header of dtype / shape / data_offsets, then the data), so a row range of a
    row-major tensor is one contiguous byte range of the file;
  * a rank of an N-sharded projection reads only its own rows' bytes
    (shard_bounds, the same split tsb.dist uses), never the whole matrix;
  * fused projections (q|k|v, gate|up) are row concatenations of the source
    modules, written straight into one device buffer (each row carries its own
    scales and biases, so concatenating rows is exact);
  * file reads go through two pinned staging buffers, so the read of one chunk
    overlaps the host-to-device copy of the previous one.

Quantization parameters come from config.json's "quantization" (or
"quantization_config") entry, with mlx-lm's per-module overrides (a dict with
its own bits / group_size, or false for a module left unquantized).
"""

from __future__ import annotations

import json
import math
import os
import struct
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass

import numpy as np
import torch

from .dist import shard_bounds

# safetensors dtype -> (torch dtype holding the same bits, bytes per element).
# Unsigned 32-bit words land in int32 (bit-identical), as every tsb weight does.
_DTYPES = {
    "BF16": (torch.bfloat16, 2), "F16": (torch.float16, 2), "F32": (torch.float32, 4), "F64": (torch.float64, 8),
    "U32": (torch.int32, 4), "I32": (torch.int32, 4), "U16": (torch.int16, 2), "I16": (torch.int16, 2),
    "U8": (torch.uint8, 1), "I8": (torch.int8, 1), "U64": (torch.int64, 8), "I64": (torch.int64, 8),
    "BOOL": (torch.bool, 1),
}
_MAX_HEADER = 100 << 20


@dataclass(frozen=True)
class TensorEntry:
    file: str
    dtype: str
    shape: tuple
    offset: int    # absolute byte offset of the data in the file
    nbytes: int

    @property
    def row_bytes(self) -> int:
        return self.nbytes // self.shape[0] if self.shape and self.shape[0] else 0


def read_header(path: str) -> dict:
    """{name: TensorEntry} of one safetensors file (the "__metadata__" entry is dropped).
    Raises ValueError on a malformed header or offsets outside the file."""
    size = os.path.getsize(path)
    with open(path, "rb") as f:
        head = f.read(8)
        if len(head) != 8:
            raise ValueError(f"{path}: not a safetensors file (shorter than 8 bytes)")
        (n,) = struct.unpack("<Q", head)
        if n > min(size - 8, _MAX_HEADER):
            raise ValueError(f"{path}: header length {n} exceeds the file")
        meta = json.loads(f.read(n))
    meta.pop("__metadata__", None)
    start = 8 + n
    out = {}
    for name, e in meta.items():
        dt = e["dtype"]
        if dt not in _DTYPES:
            raise ValueError(f"{path}: {name}: unsupported dtype {dt}")
        shape = tuple(int(s) for s in e["shape"])
        b, end = (int(v) for v in e["data_offsets"])
        nbytes = math.prod(shape) * _DTYPES[dt][1]
        if b < 0 or end - b != nbytes or start + end > size:
            raise ValueError(f"{path}: {name}: data_offsets {b}..{end} do not hold {dt}{list(shape)}")
        out[name] = TensorEntry(path, dt, shape, start + b, nbytes)
    return out


def _pread_exact(fd: int, view: np.ndarray, offset: int) -> None:
    mv = memoryview(view).cast("B")
    got = 0
    while got < len(mv):
        n = os.preadv(fd, [mv[got:]], offset + got)
        if n <= 0:
            raise OSError(f"short read at byte {offset + got}")
        got += n


class _Stager:
    """File bytes -> a device (or host) tensor through two pinned staging buffers.
    Each chunk is read by several threads at once (os.preadv releases the GIL):
    one thread's copy out of the page cache runs near 8 GB/s, a pinned
    host-to-device copy several times that."""

    def __init__(self, device, chunk: int = 32 << 20, threads: int = min(8, os.cpu_count() or 1)):
        self.pool = ThreadPoolExecutor(max_workers=threads) if threads > 1 else None
        self.threads = threads
        self.device = torch.device(device)
        self.cuda = self.device.type == "cuda"
        self.chunk = chunk
        self.bufs = [torch.empty(chunk, dtype=torch.uint8, pin_memory=self.cuda) for _ in range(2)]
        self.views = [b.numpy() for b in self.bufs]
        self.events = [None, None]
        self.turn = 0
        self.fds: dict[str, int] = {}

    def _fd(self, path: str) -> int:
        if path not in self.fds:
            self.fds[path] = os.open(path, os.O_RDONLY)
        return self.fds[path]

    def copy(self, path: str, offset: int, nbytes: int, dst: torch.Tensor, dst_off: int) -> None:
        """Bytes [offset, offset + nbytes) of `path` -> bytes [dst_off, ...) of the flat uint8 view `dst`."""
        fd = self._fd(path)
        done = 0
        while done < nbytes:
            n = min(self.chunk, nbytes - done)
            i = self.turn
            self.turn ^= 1
            if self.events[i] is not None:
                self.events[i].synchronize()   # the copy that last read this buffer has finished
            self._read(fd, self.views[i][:n], offset + done)
            dst[dst_off + done:dst_off + done + n].copy_(self.bufs[i][:n], non_blocking=self.cuda)
            if self.cuda:
                ev = torch.cuda.Event()
                ev.record(torch.cuda.current_stream(self.device))
                self.events[i] = ev
            done += n

    def _read(self, fd: int, view: np.ndarray, offset: int) -> None:
        n = len(view)
        if self.pool is None or n < (4 << 20):
            _pread_exact(fd, view, offset)
            return
        step = (-(-n // self.threads) + 4095) & ~4095
        for f in [self.pool.submit(_pread_exact, fd, view[a:a + step], offset + a) for a in range(0, n, step)]:
            f.result()

    def sync(self) -> None:
        """Wait until every copy issued so far has landed."""
        for ev in self.events:
            if ev is not None:
                ev.synchronize()

    def close(self) -> None:
        self.sync()
        for fd in self.fds.values():
            os.close(fd)
        self.fds.clear()
        if self.pool is not None:
            self.pool.shutdown()
            self.pool = None


def _flat_bytes(t: torch.Tensor) -> torch.Tensor:
    return t.view(-1).view(torch.uint8)


class Checkpoint:
    """An mlx-lm checkpoint: a directory with config.json and *.safetensors
    (indexed by model.safetensors.index.json when present), or one file."""

    def __init__(self, path: str):
        if os.path.isdir(path):
            root = path
            index = os.path.join(path, "model.safetensors.index.json")
            if os.path.exists(index):
                with open(index) as f:
                    files = sorted(set(json.load(f)["weight_map"].values()))
            else:
                files = sorted(n for n in os.listdir(path) if n.endswith(".safetensors"))
            files = [os.path.join(path, n) for n in files]
        else:
            root = os.path.dirname(os.path.abspath(path))
            files = [path]
        if not files:
            raise FileNotFoundError(f"no safetensors files under {path}")
        cfg_path = os.path.join(root, "config.json")
        self.config = {}
        if os.path.exists(cfg_path):
            with open(cfg_path) as f:
                self.config = json.load(f)
        self._stagers: dict[torch.device, _Stager] = {}
        self.tensors: dict[str, TensorEntry] = {}
        for fp in files:
            for name, e in read_header(fp).items():
                if name in self.tensors:
                    raise ValueError(f"{name} appears in both {self.tensors[name].file} and {fp}")
                self.tensors[name] = e

    def _stager(self, device) -> _Stager:
        dev = torch.device(device)
        if dev.type == "cuda" and dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        if dev not in self._stagers:
            self._stagers[dev] = _Stager(dev)
        return self._stagers[dev]

    def close(self) -> None:
        """Wait for outstanding copies, close the files and free the staging
        buffers (a later load sets them up again)."""
        for st in self._stagers.values():
            st.close()
        self._stagers.clear()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # ---------------------------------------------------------------- format

    def quantization(self, module: str):
        """{"bits", "group_size", "mode"} of a module, or None when it is not quantized."""
        q = self.config.get("quantization", self.config.get("quantization_config"))
        if not q:
            return None
        base = {"bits": q.get("bits", 4), "group_size": q.get("group_size", 64), "mode": q.get("mode", "affine")}
        per = q.get(module)
        if per is False:
            return None
        if isinstance(per, dict):
            base.update({k: per[k] for k in ("bits", "group_size", "mode") if k in per})
        return base

    def decline(self, module: str):
        """None when `module` is a linear the verify qmm takes, else the reason.
        The rule is the reference's (packed_linear.py:49-58: 4-bit affine with
        biases and no bias, N % 32 == 0, K % 128 == 0) plus this library's
        (group size 64, bf16 scales, N % 128 == 0)."""
        w, s, b = (self.tensors.get(f"{module}.{p}") for p in ("weight", "scales", "biases"))
        if w is None:
            return "no weight"
        q = self.quantization(module)
        if q is None or s is None:
            return "not quantized"
        if q["bits"] != 4 or q["mode"] != "affine":
            return f"{q['bits']}-bit {q['mode']} (only 4-bit affine)"
        if b is None:
            return "no biases"
        if f"{module}.bias" in self.tensors:
            return "has an additive bias"
        if w.dtype not in ("U32", "I32") or len(w.shape) != 2:
            return f"weight {w.dtype}{list(w.shape)} (want 2-D uint32 words)"
        n, k = w.shape[0], w.shape[1] * 8
        gs = q["group_size"]
        if gs != 64:
            return f"group size {gs} (only 64)"
        if s.shape != (n, k // gs) or b.shape != s.shape:
            return f"scales {list(s.shape)} / biases {list(b.shape)} do not match weight [{n}, {k}/{gs}]"
        if s.dtype != "BF16" or b.dtype != "BF16":
            return f"{s.dtype} scales (the kernels read bf16)"
        if n % 32 or k % 128:
            return f"N={n}, K={k} (the reference's kernels want N % 32 == 0, K % 128 == 0)"
        if n % 128:
            return f"N={n} (the verify qmm tiles 128 rows)"
        return None

    def linear_shape(self, module: str) -> tuple[int, int]:
        w = self.tensors[f"{module}.weight"]
        return w.shape[0], w.shape[1] * 8

    def quantized_linears(self) -> dict:
        """{module: None (eligible) or the reason it is declined} for every quantized linear."""
        mods = sorted({n[:-len(".scales")] for n in self.tensors if n.endswith(".scales")})
        return {m: self.decline(m) for m in mods}

    # ---------------------------------------------------------------- loading

    def load_linear(self, modules, device="cuda", world: int = 1, rank: int = 0):
        """(wq int32 [Nr, K/8], scales bf16 [Nr, K/64], biases bf16) on `device`:
        the row concatenation of `modules` (one name, or a list for a fused
        projection), or rank's row shard of it when world > 1. Raises
        ValueError if a module is declined or the K dimensions differ."""
        mods = [modules] if isinstance(modules, str) else list(modules)
        for m in mods:
            why = self.decline(m)
            if why is not None:
                raise ValueError(f"{m}: {why}")
        ks = {self.linear_shape(m)[1] for m in mods}
        if len(ks) != 1:
            raise ValueError(f"{mods}: different K {sorted(ks)}")
        k = ks.pop()
        n_total = sum(self.linear_shape(m)[0] for m in mods)
        r0, r1 = shard_bounds(n_total, world, rank) if world > 1 else (0, n_total)
        dev = torch.device(device)
        wq = torch.empty((r1 - r0, k // 8), dtype=torch.int32, device=dev)
        sc = torch.empty((r1 - r0, k // 64), dtype=torch.bfloat16, device=dev)
        bi = torch.empty_like(sc)
        dsts = {"weight": _flat_bytes(wq), "scales": _flat_bytes(sc), "biases": _flat_bytes(bi)}
        st = self._stager(dev)
        g0 = 0
        for m in mods:
            n = self.linear_shape(m)[0]
            a, b = max(r0, g0), min(r1, g0 + n)   # this module's rows inside the shard
            if a < b:
                for part, dst in dsts.items():
                    e = self.tensors[f"{m}.{part}"]
                    rb = e.row_bytes
                    st.copy(e.file, e.offset + (a - g0) * rb, (b - a) * rb, dst, (a - r0) * rb)
            g0 += n
        st.sync()
        return wq, sc, bi

    def load_tensor(self, name: str, device="cuda", dtype=None) -> torch.Tensor:
        """One tensor as stored (uint32 as int32), optionally converted to `dtype` on the device."""
        e = self.tensors[name]
        dt = _DTYPES[e.dtype][0]
        out = torch.empty(e.shape, dtype=dt, device=torch.device(device))
        if e.nbytes:
            st = self._stager(device)
            st.copy(e.file, e.offset, e.nbytes, _flat_bytes(out), 0)
            st.sync()
        return out if dtype is None or dtype == dt else out.to(dtype)


# ---------------------------------------------------------------- the decoder's layout

# Module names of a gated-q attention layer in an mlx-lm checkpoint (the
# attributes tree_verify.py:311-327 and 414-447 read: attn.q_proj ... o_proj,
# q_norm, k_norm, mlp gate/up/down, input and post-attention norms).
LAYER_NAMES = {
    "q": "self_attn.q_proj", "k": "self_attn.k_proj", "v": "self_attn.v_proj", "o": "self_attn.o_proj",
    "gate": "mlp.gate_proj", "up": "mlp.up_proj", "down": "mlp.down_proj",
    "q_norm": "self_attn.q_norm", "k_norm": "self_attn.k_norm",
    "input_norm": "input_layernorm", "post_norm": "post_attention_layernorm",
}


def _rope_field(c: dict, key: str):
    """A rope setting at the top level of the text config, or nested under
    "rope_parameters" (the newer Hugging Face / mlx-lm layout); None if absent."""
    if key in c:
        return c[key]
    return (c.get("rope_parameters") or {}).get(key)


def decoder_config(ckpt: Checkpoint, **overrides):
    """A tsb.decoder.DecoderConfig from the checkpoint's config.json (its
    "text_config" when nested). rope_theta and partial_rotary_factor are read
    at the top level or under "rope_parameters"; a config with no rope_theta in
    either place is refused (ValueError) rather than given a default base, and a
    missing partial_rotary_factor means full rotary (1.0), its Hugging Face
    meaning. rope_dims = head_dim * partial_rotary_factor."""
    from .decoder import DecoderConfig

    c = ckpt.config.get("text_config", ckpt.config)
    d = c.get("head_dim", c["hidden_size"] // c["num_attention_heads"])
    theta = overrides.get("rope_base", _rope_field(c, "rope_theta"))
    if theta is None:
        raise ValueError("config has no rope_theta (top level or rope_parameters); pass rope_base=")
    factor = _rope_field(c, "partial_rotary_factor")
    kw = dict(layers=c["num_hidden_layers"], hidden=c["hidden_size"], hq=c["num_attention_heads"],
              hkv=c.get("num_key_value_heads", c["num_attention_heads"]), d=d, inter=c["intermediate_size"],
              eps=c.get("rms_norm_eps", 1e-6), rope_dims=int(d * (1.0 if factor is None else factor)),
              rope_base=float(theta))
    kw.update(overrides)
    return DecoderConfig(**kw)


# Where mlx-lm checkpoints keep the text model's layers: plain decoders under
# "model.layers", multimodal wrappers (e.g. qwen3_5) under the language model.
LAYER_PREFIXES = ("model.layers", "language_model.model.layers", "model.language_model.layers")


def decoder_layers(ckpt: Checkpoint, cfg, indices=None, prefix: str | None = None, final_norm: str | None = None,
                   device="cuda", names: dict | None = None):
    """(layers, final_norm) for tsb.decoder.VerifyDecoder, read from `ckpt`:
    q|k|v fused into one qkv projection, gate|up into gate_up, the norms as
    bf16. indices: the layer numbers to load (default: every layer with a
    q_proj, i.e. the full-attention layers of a hybrid model). prefix: where the
    layers live (default: the first of LAYER_PREFIXES that holds a q_proj);
    final_norm: the final norm's module (default: the prefix's ".norm")."""
    nm = dict(LAYER_NAMES, **(names or {}))

    def layer_numbers(pfx):
        return sorted(int(n.split(".")[len(pfx.split("."))]) for n in ckpt.tensors
                      if n.startswith(pfx + ".") and n.endswith(nm["q"] + ".weight"))

    if prefix is None:
        prefix = next((p for p in LAYER_PREFIXES if layer_numbers(p)), None)
        if prefix is None:
            raise ValueError(f"no layer with a {nm['q']} under any of {LAYER_PREFIXES}; pass prefix=")
    if final_norm is None:
        final_norm = prefix[: -len(".layers")] + ".norm" if prefix.endswith(".layers") else "model.norm"
    if indices is None:
        indices = layer_numbers(prefix)
        if not indices:
            raise ValueError(f"no layer with a {nm['q']} under {prefix!r}")
    layers = []
    for i in indices:
        p = f"{prefix}.{i}."
        qkv_rows = sum(ckpt.linear_shape(p + nm[x])[0] for x in ("q", "k", "v"))
        if qkv_rows != cfg.qkv_rows:
            raise ValueError(f"layer {i}: q|k|v has {qkv_rows} rows, the config wants {cfg.qkv_rows}")
        layers.append({
            "qkv": ckpt.load_linear([p + nm["q"], p + nm["k"], p + nm["v"]], device),
            "o": ckpt.load_linear(p + nm["o"], device),
            "gate_up": ckpt.load_linear([p + nm["gate"], p + nm["up"]], device),
            "down": ckpt.load_linear(p + nm["down"], device),
            **{key: ckpt.load_tensor(p + nm[key] + ".weight", device, torch.bfloat16)
               for key in ("q_norm", "k_norm", "input_norm", "post_norm")},
        })
    return layers, ckpt.load_tensor(final_norm + ".weight", device, torch.bfloat16)
