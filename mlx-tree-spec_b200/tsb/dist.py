"""N-sharded (column-parallel) quantized matmul across the GPUs of one box.

The reference runs on one device and has no collectives. The B200 build adds
one strategy, per its target: every 4-bit weight (N, K) is split by output
rows over G ranks (rank r holds rows [r*N/G, (r+1)*N/G) of w, scales and
biases, so each shard is itself a valid MLX-format weight); x is replicated;
each rank computes its (M, N/G) slice and, where a layer's full output is
needed, the slices are reassembled with one NCCL all-gather over NVLink.

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

    def forward_into(self, x, wq, s, b, out):
        """x (M, K) contiguous; (wq, s, b) this rank's shard; out (M, N) full."""
        import torch.distributed as dist

        m = x.shape[0]
        ns = wq.shape[0]
        local, gathered = self._buf(m, ns, out.dtype, out.device)
        self.local_op(x, wq, s, b, local, ns)
        dist.all_gather_into_tensor(gathered.view(self.world * m, ns), local, group=self.group)
        return gather_relayout(gathered, out)

    def forward(self, x, wq, s, b):
        k = x.shape[-1]
        x2 = x.reshape(-1, k).contiguous()
        out = torch.empty(x2.shape[0], wq.shape[0] * self.world, dtype=x.dtype, device=x.device)
        self.forward_into(x2, wq, s, b, out)
        return out.reshape(*x.shape[:-1], out.shape[-1])
