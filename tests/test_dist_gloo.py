"""Head-parallel host logic on CPU: two gloo ranks in child processes.

Covers what a multi-GPU job does on the host: the head partition, the
broadcast of rank 0's 128-byte NCCL id, the max-over-ranks timing reduction
the bench uses, and the all-gather layout contract (rank r's head block lands
at heads [r*H/N, (r+1)*H/N)), checked with gloo's all_gather standing in for
NCCL.  A rank that fails raises in its process and the parent sees the exit.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ltxattn import dist as ldist


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        from datetime import timedelta
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        # head partition
        begin, count = ldist.head_block(32, world, rank)
        assert count == 32 // world and begin == rank * count
        # id exchange (a fixed fake id: no NCCL needed on CPU)
        fake = bytes(range(128))
        got = ldist.exchange_unique_id(make_id=fake if rank == 0 else None)
        assert got == fake
        # max over ranks
        m = ldist.max_over_ranks([1.0 + rank, 10.0 - rank])
        assert m == [float(world), 10.0]
        # gather layout: each rank holds its heads; all_gather per batch as the C entry does
        B, T, D = 2, 5, 4
        local = torch.arange(B * count * T * D, dtype=torch.float32).reshape(B, count, T, D) + 1000 * rank
        blocks = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(blocks, local)
        full = ldist.gather_layout(blocks)
        assert full.shape == (B, 32, T, D)
        for r in range(world):
            b0, c = ldist.head_block(32, world, r)
            assert torch.equal(full[:, b0:b0 + c], blocks[r])
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e)))
        raise


def test_two_gloo_ranks():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    results = dict(q.get(timeout=5) for _ in range(world))
    assert all(p.exitcode == 0 for p in procs), results
    assert results == {0: "ok", 1: "ok"}


def test_head_block_rejects_uneven_split():
    with pytest.raises(Exception):
        ldist.head_block(32, 3, 0)
    with pytest.raises(Exception):
        ldist.head_block(32, 2, 2)
