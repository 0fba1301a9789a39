"""ltxattn_fwd_gather on two GPUs: each rank computes its head block and its
epilogue stores every output tile into both ranks' outputs over NVLink (the
all-gather fused into the attention), with bounded entry and arrival
handshakes between the devices.

Every rank's gathered output must equal, bit for bit, the same head-block calls
made on one device (ltxattn_fwd with head_begin / head_count: the same plan, so
split KV ranges and their combine, which stores the split rows to the peers,
are exercised: 6 and 52 units per rank here), across several calls (the epoch
handshake) with changing data.  Runs as
two spawned processes (gloo for the host exchange); skipped with fewer than two
GPUs."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, shape, results):
    import torch.distributed as dist
    from datetime import timedelta
    from ltxattn import AttentionBackend, Rotary, device_status, inputs
    from ltxattn.dist import FusedHeadGather, head_block
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    reported = False
    try:
        B, H, T, D = shape
        dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to("cuda", torch.bfloat16)
        q = dev(inputs.seeded_tensor(501, (B, H, T, D), rmsnorm=True))
        k = dev(inputs.seeded_tensor(502, (B, H, T, D), rmsnorm=True))
        v = dev(inputs.seeded_tensor(503, (B, H, T, D)))
        grid = {700: (5, 10, 14), 3120: (13, 12, 20)}[T]  # frames x height x width = T tokens
        cos, sin = inputs.rope3d_grid(*grid, D)
        rot = Rotary(dev(cos), dev(sin))
        g = FusedHeadGather((B, H, T, D))
        ok = True
        for call in range(3):
            vv = v * (call + 1)  # other data every call: stale tiles would show
            g.out.fill_(7.0)
            out = g.run(q, k, vv, q_rotary=rot)
            torch.cuda.synchronize()
            ref = torch.empty_like(out)
            for r in range(world):
                h0, hc = head_block(H, world, r)
                AttentionBackend.attention(q, k, vv, q_rotary=rot, head_begin=h0, head_count=hc, out=ref)
            torch.cuda.synchronize()
            ok = ok and torch.equal(out, ref)
            dist.barrier()  # both ranks compared before the next call overwrites
        status = device_status(clear=True)
        g.close()
        results.put((rank, bool(ok), int(status)))
        reported = True
    finally:
        if not reported:
            results.put((rank, False, -1))  # the parent learns of a failure at once
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("shape", [(1, 4, 700, 128), (1, 8, 3120, 128)])
def test_fused_gather_matches_the_block_calls_on_two_gpus(shape):
    world = 2
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, shape, results)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        r, ok, status = results.get(timeout=300)
        got[r] = (ok, status)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(world):
        assert got[r] == (True, 0), f"rank {r}: bit-identical {got[r][0]}, device status {got[r][1]}"


def _outproj_rank_main(rank, world, port, shape, results):
    import torch.distributed as dist
    from datetime import timedelta
    from ltxattn import device_status
    from ltxattn import dist as ldist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    reported = False
    try:
        m, n, K = shape
        k = K // world
        g = torch.Generator(device="cuda").manual_seed(11)  # the same tensors on every rank
        merged = torch.randn((m, K), generator=g, device="cuda").to(torch.bfloat16)
        W = (torch.randn((n, K), generator=g, device="cuda") / 64).to(torch.bfloat16)
        b = (torch.randn(n, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
        w_block = W[:, rank * k:(rank + 1) * k]
        uid = ldist.exchange_unique_id()
        hg = ldist.HeadGather(world, rank, uid, rank)
        fo = ldist.FusedOutProject(m, n)
        ok = True
        for call in range(3):
            x_local = (merged[:, rank * k:(rank + 1) * k] * (call + 1)).contiguous()
            ref = hg.out_project(x_local, w_block, b)  # GEMM, NCCL all-reduce, bias and rounding
            fo.out.fill_(3.0)
            got = fo.run(x_local, w_block, b)
            torch.cuda.synchronize()
            # two ranks: the fp32 sum of two partials is the same in either order
            ok = ok and torch.equal(got, ref)
        status = device_status(clear=True)
        fo.close()
        hg.close()
        results.put((rank, bool(ok), int(status)))
        reported = True
    finally:
        if not reported:
            results.put((rank, False, -1))
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("shape", [(300, 512, 1024), (3120, 4096, 4096)])
def test_fused_out_project_matches_the_nccl_all_reduce_on_two_gpus(shape):
    # ltxattn_out_project_fused (partial rows stored into their owners' planes by the
    # GEMM's epilogue, owners reduce in rank order and store into every output)
    # against ltxattn_out_project_allreduce on the same inputs: bit-identical
    world = 2
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_outproj_rank_main, args=(r, world, port, shape, results)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        r, ok, status = results.get(timeout=300)
        got[r] = (ok, status)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(world):
        assert got[r] == (True, 0), f"rank {r}: bit-identical {got[r][0]}, device status {got[r][1]}"
