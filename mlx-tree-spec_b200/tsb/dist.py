"""N-sharded (column-parallel) quantized matmul across the GPUs of one box.

The reference runs on one device and has no collectives. The B200 build adds
one strategy, per its target: every 4-bit weight (N, K) is split by output
rows over G ranks (rank r holds rows [r*N/G, (r+1)*N/G) of w, scales and
biases, so each shard is itself a valid MLX-format weight); x is replicated;
each rank computes its (M, N/G) slice and every rank ends with the full
(M, N) output.

Two forms:
  GatheredQMM  any M: one kernel per rank (the verify kernel at M <= 128, the
               prefill GEMM above) computes its slice and stores each finished
               tile into every rank's output over NVLink (peer memory from
               torch symmetric memory), exchanging completion flags itself
               (tsb_qmm_w4g64_gather): the transfer overlaps the matmul and no
               separate collective runs.
  ShardedQMM   any M: the shard's matmul, then NCCL all-gathers and a
               relayout into the caller's buffer (optionally block by block of
               rows, overlapped with the next block's matmul).

Every rank takes the same collective steps in the same order.
"""

from __future__ import annotations

import torch


def shard_bounds(n: int, world: int, rank: int, align: int = 128) -> tuple[int, int]:
    """Row range of `rank`'s shard; N/world must be a multiple of `align` (the
    kernel's row tile) so every shard stays on the fast path."""
    if n % world:
        raise ValueError(f"N={n} not divisible by world={world}")
    ns = n // world
    if ns % align:
        raise ValueError(f"shard of {ns} rows is not a multiple of {align}")
    return rank * ns, (rank + 1) * ns


def shard_weight(w, scales, biases, world: int, rank: int):
    a, b = shard_bounds(w.shape[0], world, rank)
    return w[a:b].contiguous(), scales[a:b].contiguous(), biases[a:b].contiguous()


def gather_relayout(gathered: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """[G, M, N/G] rank-major slices -> out [M, N] (column block g from rank g)."""
    g, m, ns = gathered.shape
    out.view(m, g, ns).copy_(gathered.permute(1, 0, 2))
    return out


class ShardedQMM:
    """y = x @ W.T with W N-sharded over the process group."""

    def __init__(self, world: int, rank: int, group=None, local_op=None):
        self.world, self.rank, self.group = world, rank, group
        self._bufs: dict = {}
        self._streams: dict = {}
        # local_op(x2, wq, s, b, y, ldy): the shard's matmul (the CUDA kernel by
        # default; tests substitute a CPU stand-in to check the host logic).
        if local_op is None:
            from .ops import quantized_matmul_into

            local_op = quantized_matmul_into
        self.local_op = local_op

    def _buf(self, m, ns, dtype, device):
        key = (m, ns, dtype, str(device))
        b = self._bufs.get(key)
        if b is None:
            b = (torch.empty(m, ns, dtype=dtype, device=device),
                 torch.empty(self.world, m, ns, dtype=dtype, device=device))
            self._bufs[key] = b
        return b

    def _comm_stream(self, device):
        st = self._streams.get(str(device))
        if st is None:
            st = torch.cuda.Stream(device=device)
            self._streams[str(device)] = st
        return st

    def forward_into(self, x, wq, s, b, out, chunks: int = 1):
        """x (M, K) contiguous; (wq, s, b) this rank's shard; out (M, N) full.

        chunks > 1 (M a multiple of it): the shard's matmul runs `chunks` row
        blocks of x in turn, and each block's all-gather and re-layout into
        `out` run on a side stream while the next block computes (on CUDA; on
        the CPU the blocks run in order), so the collective overlaps compute."""
        import torch.distributed as dist

        m = x.shape[0]
        ns = wq.shape[0]
        local, gathered = self._buf(m, ns, out.dtype, out.device)
        if chunks <= 1 or m % chunks:
            self.local_op(x, wq, s, b, local, ns)
            dist.all_gather_into_tensor(gathered.view(self.world * m, ns), local, group=self.group)
            return gather_relayout(gathered, out)
        c = m // chunks
        blocks = gathered.view(chunks, self.world, c, ns)  # one contiguous [world, c, ns] per block
        if not x.is_cuda:
            for i in range(chunks):
                self.local_op(x[i * c:(i + 1) * c], wq, s, b, local[i * c:(i + 1) * c], ns)
                dist.all_gather_into_tensor(blocks[i].view(self.world * c, ns), local[i * c:(i + 1) * c],
                                            group=self.group)
                gather_relayout(blocks[i], out[i * c:(i + 1) * c])
            return out
        cur = torch.cuda.current_stream(x.device)
        comm = self._comm_stream(x.device)
        comm.wait_stream(cur)  # out and the buffers are free once earlier work on the stream is done
        for i in range(chunks):
            self.local_op(x[i * c:(i + 1) * c], wq, s, b, local[i * c:(i + 1) * c], ns)
            ev = torch.cuda.Event()
            ev.record(cur)
            with torch.cuda.stream(comm):
                comm.wait_event(ev)
                dist.all_gather_into_tensor(blocks[i].view(self.world * c, ns), local[i * c:(i + 1) * c],
                                            group=self.group)
                gather_relayout(blocks[i], out[i * c:(i + 1) * c])
        cur.wait_stream(comm)
        return out

    def forward(self, x, wq, s, b):
        k = x.shape[-1]
        x2 = x.reshape(-1, k).contiguous()
        out = torch.empty(x2.shape[0], wq.shape[0] * self.world, dtype=x.dtype, device=x.device)
        self.forward_into(x2, wq, s, b, out)
        return out.reshape(*x.shape[:-1], out.shape[-1])


# Words of a GatheredQMM signal block (the kernel uses 2 * world + 3 of them).
SIG_WORDS = 64


class GatheredQMM:
    """y = x @ W.T with W N-sharded over the process group, gathered inside the
    kernel: rank r's kernel writes its columns into every rank's y.

    Outputs must come from out_buffer(m, n) (symmetric memory: every rank
    holds the same buffer and can address its peers'). One signal block per
    instance; every rank makes the same sequence of calls on one stream."""

    def __init__(self, world: int, rank: int, group=None, device=None):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        from . import _lib

        if world > _lib.TSB_MAX_GATHER_RANKS:
            raise ValueError(f"world {world} > {_lib.TSB_MAX_GATHER_RANKS}")
        self.world, self.rank = world, rank
        self.group = group if group is not None else dist.group.WORLD
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self._symm = symm_mem
        sig = symm_mem.empty(SIG_WORDS, dtype=torch.int32, device=self.device)
        sig.zero_()
        self._sig = sig
        self._sig_ptrs = list(symm_mem.rendezvous(sig, self.group).buffer_ptrs)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # every block is zero before any rank's first call
        self._outs: dict = {}

    def out_buffer(self, m: int, n: int, dtype=torch.bfloat16) -> torch.Tensor:
        """The (m, n) output buffer of this shape (allocated once, collectively:
        every rank must ask for the same shapes in the same order)."""
        key = (m, n, dtype)
        hit = self._outs.get(key)
        if hit is None:
            from . import _lib

            t = self._symm.empty(m, n, dtype=dtype, device=self.device)
            ptrs = list(self._symm.rendezvous(t, self.group).buffer_ptrs)
            g = _lib.GatherT()
            g.world, g.rank = self.world, self.rank
            for p in range(self.world):
                g.y[p] = ptrs[p]
                g.sig[p] = self._sig_ptrs[p]
            hit = (t, g)
            self._outs[key] = hit
        return hit[0]

    def forward_into(self, x, wq, s, b, out):
        """x (M, K) contiguous; (wq, s, b) this rank's shard; out from out_buffer."""
        import ctypes

        from . import _lib
        from .ops import _ptr, _stream, qmm_workspace

        m, k = x.shape
        ns = wq.shape[0]
        hit = self._outs.get((out.shape[0], out.shape[1], out.dtype))
        if hit is None or hit[0].data_ptr() != out.data_ptr():
            raise ValueError("out must come from GatheredQMM.out_buffer")
        lib = _lib.load()
        ws = qmm_workspace(lib.tsb_qmm_workspace_bytes(m, ns, k), x.device)
        st = lib.tsb_qmm_w4g64_gather(_ptr(x), _ptr(wq), _ptr(s), _ptr(b), m, ns, k, out.shape[1],
                                      ctypes.byref(hit[1]), _ptr(ws), ws.numel(), _stream(x))
        if st != _lib.TSB_OK:
            raise _lib.TSBError(st, "tsb_qmm_w4g64_gather")
        return out

    def forward(self, x, wq, s, b):
        """x (..., K) -> the gathered output (..., N) in this instance's buffer
        for the shape (overwritten by the next call of the same shape)."""
        k = x.shape[-1]
        x2 = x.reshape(-1, k).contiguous()
        out = self.out_buffer(x2.shape[0], wq.shape[0] * self.world, x.dtype)
        self.forward_into(x2, wq, s, b, out)
        return out.reshape(*x.shape[:-1], out.shape[-1])
