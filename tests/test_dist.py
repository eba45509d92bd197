"""Host logic of the N-sharded qmm on world_size-2 gloo ranks (CPU).

The shard's local matmul is replaced by the oracle (a CPU stand-in injected by
the test) so that the sharding, the collective and the re-layout are checked
without a GPU."""

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import bf16, gen, qmm


def _worker(rank, world, port, ret):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from tsb.dist import ShardedQMM, shard_weight

        rng = np.random.default_rng(42)
        m, n, k = 5, 512, 256
        x = gen.x_bf16(rng, m, k)
        wq, s, b = gen.weights_w4g64(rng, n, k)
        wt = torch.from_numpy(wq.view(np.int32))
        st, bt = bf16.to_torch_bf16(s), bf16.to_torch_bf16(b)
        ws, ss, bs = shard_weight(wt, st, bt, world, rank)

        def cpu_op(x2, wq_, s_, b_, y, ldy):
            r = qmm.qmm(bf16.from_torch_bf16(x2), wq_.numpy().view(np.uint32), bf16.from_torch_bf16(s_),
                        bf16.from_torch_bf16(b_))
            y.copy_(torch.from_numpy(r.astype(np.float32)).to(y.dtype))

        op = ShardedQMM(world, rank, local_op=cpu_op)
        y = op.forward(bf16.to_torch_bf16(x), ws, ss, bs)
        ref = qmm.qmm(x, wq, s, b)
        err = float(np.max(np.abs(y.float().numpy() - ref)))
        ok = err <= 1e-2 * np.max(np.abs(ref))
        # the chunked form (row blocks gathered one by one) gives the same output
        x6 = gen.x_bf16(rng, 6, k)
        yc = torch.empty(6, n, dtype=torch.bfloat16)
        op.forward_into(bf16.to_torch_bf16(x6), ws, ss, bs, yc, chunks=3)
        y1 = torch.empty(6, n, dtype=torch.bfloat16)
        op.forward_into(bf16.to_torch_bf16(x6), ws, ss, bs, y1)
        ret[rank] = ok and torch.equal(yc, y1)
    finally:
        dist.destroy_process_group()


def test_sharded_qmm_gloo_world2():
    world = 2
    port = 29500 + (os.getpid() % 1000)
    with mp.get_context("spawn").Manager() as man:
        ret = man.dict()
        mp.spawn(_worker, args=(world, port, ret), nprocs=world, join=True)
        assert ret.get(0) and ret.get(1)


def test_shard_bounds():
    from tsb.dist import shard_bounds

    assert shard_bounds(34816, 8, 3) == (13056, 17408)
    assert shard_bounds(6144, 8, 7) == (5376, 6144)
    with pytest.raises(ValueError):
        shard_bounds(5120, 3, 0)
    with pytest.raises(ValueError):
        shard_bounds(5120, 16, 0)  # 320-row shards are not multiples of 128


def test_gather_relayout():
    from tsb.dist import gather_relayout

    g = torch.arange(2 * 3 * 4, dtype=torch.float32).reshape(2, 3, 4)
    out = torch.empty(3, 8)
    gather_relayout(g, out)
    assert torch.equal(out[:, :4], g[0]) and torch.equal(out[:, 4:], g[1])
