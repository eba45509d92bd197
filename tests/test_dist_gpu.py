"""Tensor-parallel qmm on 2, 4 and 8 GPUs. The output gathered inside the
kernel (tsb_qmm_w4g64_gather; the verify kernel and, past M = 128, the prefill
GEMM): each rank's output holds every rank's columns, bit-identical to each
shard's single-GPU result, across repeated calls into the same buffer, eager
and replayed from a CUDA graph. The prefill (M = 4096) with NCCL all-gathers
overlapped against the row blocks' matmuls (ShardedQMM chunks): bit-identical
to the single-GPU results of the same row blocks.

Each world size needs that many GPUs (skipped otherwise): ranks that wait on
one another never share a GPU."""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import sys
    from datetime import timedelta

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "mlx-tree-spec_b200"))
    import torch.distributed as dist

    import tsb
    from tsb import dist as tdist
    from tsb import ops

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        gq = tdist.GatheredQMM(world, rank)
        errors = []
        for (m, n, k) in [(16, 6144, 5120), (1, 1024, 1024), (64, 2048, 2560), (128, 1024, 640), (33, 3072, 1536),
                          (4096, 34816 // 8 * world, 5120), (300, 1024, 640), (4096, 2560 * world, 1024)]:
            g = torch.Generator(device="cuda").manual_seed(1000 + m + n)
            wq, s, b = tsb.quantize(torch.randn(n, k, device="cuda", generator=g) * 0.02)
            x = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
            shards = [tdist.shard_weight(wq, s, b, world, r) for r in range(world)]
            ref = torch.cat([ops.quantized_matmul(x, *sh) for sh in shards], dim=1)
            out = gq.out_buffer(m, n)
            for rep in range(3):
                out.fill_(0)
                gq.forward_into(x, *shards[rank], out)
                torch.cuda.synchronize()
                if not torch.equal(out, ref):
                    errors.append(f"eager {m}x{n}x{k} rep {rep}")
            # captured: several calls into the same buffer per replay
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=side):
                    for _ in range(4):
                        gq.forward_into(x, *shards[rank], out)
            torch.cuda.current_stream().wait_stream(side)
            for rep in range(3):
                graph.replay()
                torch.cuda.synchronize()
                if not torch.equal(out, ref):
                    errors.append(f"graph {m}x{n}x{k} rep {rep}")
            del graph
        # prefill: N-sharded M = 4096, all-gathered block by block behind the compute
        sq = tdist.ShardedQMM(world, rank)
        for (m, n, k) in [(4096, 34816 // 8 * world, 5120), (4096, 5120 // 8 * world, 17408 // 4)]:
            g = torch.Generator(device="cuda").manual_seed(2000 + n + k)
            wq, s, b = tsb.quantize(torch.randn(n, k, device="cuda", generator=g) * 0.02)
            x = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
            shards = [tdist.shard_weight(wq, s, b, world, r) for r in range(world)]
            for chunks in (1, 4):
                # each row block is one single-GPU call of M / chunks rows (the
                # prefill GEMM's split of its last wave depends on M)
                c = m // chunks
                ref = torch.cat([torch.cat([ops.quantized_matmul(x[i * c:(i + 1) * c], *sh) for sh in shards], dim=1)
                                 for i in range(chunks)], dim=0)
                out = torch.zeros(m, n, dtype=torch.bfloat16, device="cuda")
                sq.forward_into(x, *shards[rank], out, chunks=chunks)
                torch.cuda.synchronize()
                if not torch.equal(out, ref):
                    errors.append(f"prefill {m}x{n}x{k} chunks {chunks}")
        status = tsb._lib.load().tsb_device_status(None, 0)
        torch.cuda.synchronize()
        dist.barrier()
        q.put((rank, errors, status))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, [repr(e)], -1))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_gathered_qmm(world):
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, errors, status in sorted(results):
        assert not errors, (rank, errors)
        assert status == 0, (rank, status)
