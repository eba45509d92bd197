"""The checkpoint loader on world_size-2 gloo ranks (CPU): each rank reads only
its row shard of a fused q|k|v projection, and an all-gather of the shards
rebuilds the full projection bit for bit (the N-sharded qmm's weights)."""

import os

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ckpt_util import write_checkpoint
from oracle import gen

MODS = {"l.q": 384, "l.k": 256, "l.v": 128}   # 768 rows: shards of 384 straddle q|k


def _worker(rank, world, port, path, ret):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from tsb.checkpoint import Checkpoint

        ck = Checkpoint(path)
        mods = list(MODS)
        mine = ck.load_linear(mods, "cpu", world=world, rank=rank)
        ok = True
        for part, full in zip(mine, ck.load_linear(mods, "cpu")):
            bits = part.view(torch.int32)   # gloo gathers no 16-bit types: bf16 pairs as int32 words
            got = [torch.empty_like(bits) for _ in range(world)]
            dist.all_gather(got, bits.contiguous())
            want = full.view(torch.int32)
            ok = ok and part.shape[0] == full.shape[0] // world and torch.equal(torch.cat(got), want)
        ret[rank] = ok
    finally:
        dist.destroy_process_group()


def test_sharded_load_gloo_world2(tmp_path):
    rng = np.random.default_rng(9)
    tensors = {}
    for name, n in MODS.items():
        wq, s, b = gen.weights_w4g64(rng, n, 256)
        tensors[f"{name}.weight"] = torch.from_numpy(wq.view(np.int32))
        tensors[f"{name}.scales"] = torch.from_numpy(s.view(np.int16)).view(torch.bfloat16)
        tensors[f"{name}.biases"] = torch.from_numpy(b.view(np.int16)).view(torch.bfloat16)
    write_checkpoint(str(tmp_path), tensors, {"quantization": {"group_size": 64, "bits": 4}})
    world = 2
    port = 30500 + (os.getpid() % 1000)
    with mp.get_context("spawn").Manager() as man:
        ret = man.dict()
        mp.spawn(_worker, args=(world, port, str(tmp_path), ret), nprocs=world, join=True)
        assert ret.get(0) and ret.get(1)
