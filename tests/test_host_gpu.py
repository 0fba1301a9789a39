"""ltxattn.host.HostAttention: the fused attention with q, k, v and the output in
pinned host memory, pipelined by head block over three streams (copies in,
ltxattn_fwd per block, copies out).  Its output must be bit-identical to the
same head-block calls on device buffers (and stay so across repeated runs on
the same staging buffers), and to one call over all heads when no call splits
a KV range."""
import numpy as np
import pytest
import torch

from ltxattn import AttentionBackend, Rotary, device_status, inputs
from ltxattn.host import HostAttention, tapered_blocks

pytestmark = pytest.mark.gpu


def _case(H=8, T=3120, D=128):
    q = inputs.seeded_tensor(81, (1, H, T, D), rmsnorm=True)
    k = inputs.seeded_tensor(82, (1, H, T, D), rmsnorm=True)
    v = inputs.seeded_tensor(83, (1, H, T, D))
    cos, sin = inputs.rope3d_grid(13, 12, 20, D)
    return q, k, v, Rotary(dev(cos), dev(sin))


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda", torch.bfloat16)


def host(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16).pin_memory()


def test_host_pipeline_is_bit_identical_to_the_device_block_calls():
    q, k, v, rot = _case()
    dq, dk, dv = dev(q), dev(k), dev(v)
    blocks = ((0, 3), (3, 3), (6, 2))
    want = torch.empty_like(dq)
    for h0, hc in blocks:
        AttentionBackend.attention(dq, dk, dv, q_rotary=rot, head_begin=h0, head_count=hc, out=want)
    one, _ = AttentionBackend.attention(dq, dk, dv, q_rotary=rot)
    hq, hk, hv = host(q), host(k), host(v)
    hout = torch.empty(q.shape, dtype=torch.bfloat16).pin_memory()
    ha = HostAttention(torch.empty_like(dq), torch.empty_like(dq), torch.empty_like(dq), q_rotary=rot,
                       chunks=3)  # blocks of 3, 3 and 2 heads
    assert [(h0, hc) for h0, hc in ha.blocks] == list(blocks)
    for _ in range(2):  # the staging buffers are reused
        hout.zero_()
        ha.run(hq, hk, hv, hout)
        torch.cuda.synchronize()
        assert torch.equal(hout, want.cpu())
    # against one call over all heads: the planner may split the block calls'
    # KV ranges differently (fp32 partials), so within the bf16 tolerance
    diff = (hout.float() - one.cpu().float()).abs()
    assert diff.max().item() <= 2e-2
    assert (diff.norm() / one.float().norm().cpu()).item() <= 1e-2
    assert device_status(clear=True) == 0


def test_host_pipeline_without_splits_is_bit_identical_to_one_call():
    q, k, v, rot = _case()
    dq, dk, dv = dev(q), dev(k), dev(v)
    one, _ = AttentionBackend.attention(dq, dk, dv, q_rotary=rot, num_splits=1)
    hout = torch.empty(q.shape, dtype=torch.bfloat16).pin_memory()
    ha = HostAttention(torch.empty_like(dq), torch.empty_like(dq), torch.empty_like(dq), q_rotary=rot,
                       chunks=4, num_splits=1)
    ha.run(host(q), host(k), host(v), hout)
    torch.cuda.synchronize()
    assert torch.equal(hout, one.cpu())


def test_host_pipeline_with_a_key_mask():
    B, H, Lq, Lk, D = 1, 4, 500, 1024, 64
    q = inputs.seeded_tensor(84, (B, H, Lq, D), rmsnorm=True)
    k = inputs.seeded_tensor(85, (B, H, Lk, D), rmsnorm=True)
    v = inputs.seeded_tensor(86, (B, H, Lk, D))
    m = torch.zeros((B, Lk), dtype=torch.uint8)
    m[:, :94] = 1
    md = m.cuda()
    want = torch.empty((B, H, Lq, D), device="cuda", dtype=torch.bfloat16)
    for h in range(H):  # the block calls HostAttention makes (chunks=4: one head each)
        AttentionBackend.attention(dev(q), dev(k), dev(v), key_mask=md, head_begin=h, head_count=1, out=want)
    hout = torch.empty((B, H, Lq, D), dtype=torch.bfloat16).pin_memory()
    ha = HostAttention(dev(q).zero_(), dev(k).zero_(), dev(v).zero_(), key_mask=md, chunks=4)
    ha.run(host(q), host(k), host(v), hout)
    torch.cuda.synchronize()
    assert torch.equal(hout, want.cpu())


def test_host_pipeline_with_tapered_blocks():
    # explicit head-block sizes (the tapered schedule the benchmark uses: large
    # blocks first, a small last block): bit-identical to the same block calls
    q, k, v, rot = _case()
    dq, dk, dv = dev(q), dev(k), dev(v)
    sizes = tapered_blocks(8)
    assert sizes == [4, 2, 2]
    want = torch.empty_like(dq)
    h0 = 0
    for hc in sizes:
        AttentionBackend.attention(dq, dk, dv, q_rotary=rot, head_begin=h0, head_count=hc, out=want)
        h0 += hc
    hout = torch.empty(q.shape, dtype=torch.bfloat16).pin_memory()
    ha = HostAttention(torch.empty_like(dq), torch.empty_like(dq), torch.empty_like(dq), q_rotary=rot, blocks=sizes)
    assert [(b0, bc) for b0, bc in ha.blocks] == [(0, 4), (4, 2), (6, 2)]
    ha.run(host(q), host(k), host(v), hout)
    torch.cuda.synchronize()
    assert torch.equal(hout, want.cpu())
    with pytest.raises(Exception):
        HostAttention(torch.empty_like(dq), torch.empty_like(dq), torch.empty_like(dq), blocks=[4, 2])  # sums to 6
    assert device_status(clear=True) == 0
