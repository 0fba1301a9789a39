"""ltxattn.host.HostAttention: the fused attention with q, k, v and the output in
pinned host memory, pipelined by head block over three streams (copies in,
ltxattn_fwd per block, copies out).  Its output must be bit-identical to one
device call over all heads, and stay so across repeated runs on the same
staging buffers."""
import numpy as np
import pytest
import torch

from ltxattn import AttentionBackend, Rotary, device_status, inputs
from ltxattn.host import HostAttention

pytestmark = pytest.mark.gpu


def test_host_pipeline_is_bit_identical_to_one_device_call():
    B, H, T, D = 1, 8, 3120, 128
    q = inputs.seeded_tensor(81, (B, H, T, D), rmsnorm=True)
    k = inputs.seeded_tensor(82, (B, H, T, D), rmsnorm=True)
    v = inputs.seeded_tensor(83, (B, H, T, D))
    cos, sin = inputs.rope3d_grid(13, 12, 20, D)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to("cuda", torch.bfloat16)
    rot = Rotary(dev(cos), dev(sin))
    want, _ = AttentionBackend.attention(dev(q), dev(k), dev(v), q_rotary=rot)
    host = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16).pin_memory()
    hq, hk, hv = host(q), host(k), host(v)
    hout = torch.empty((B, H, T, D), dtype=torch.bfloat16).pin_memory()
    ha = HostAttention(torch.empty_like(want), torch.empty_like(want), torch.empty_like(want), q_rotary=rot,
                       chunks=3)  # blocks of 3, 3 and 2 heads
    for _ in range(2):
        hout.zero_()
        ha.run(hq, hk, hv, hout)
        torch.cuda.synchronize()
        assert torch.equal(hout, want.cpu())
    assert device_status(clear=True) == 0


def test_host_pipeline_with_a_key_mask():
    B, H, Lq, Lk, D = 1, 4, 500, 1024, 64
    q = inputs.seeded_tensor(84, (B, H, Lq, D), rmsnorm=True)
    k = inputs.seeded_tensor(85, (B, H, Lk, D), rmsnorm=True)
    v = inputs.seeded_tensor(86, (B, H, Lk, D))
    m = torch.zeros((B, Lk), dtype=torch.uint8)
    m[:, :94] = 1
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to("cuda", torch.bfloat16)
    md = m.cuda()
    want, _ = AttentionBackend.attention(dev(q), dev(k), dev(v), key_mask=md)
    host = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16).pin_memory()
    hout = torch.empty((B, H, Lq, D), dtype=torch.bfloat16).pin_memory()
    ha = HostAttention(dev(q).zero_(), dev(k).zero_(), dev(v).zero_(), key_mask=md, chunks=4)
    ha.run(host(q), host(k), host(v), hout)
    torch.cuda.synchronize()
    assert torch.equal(hout, want.cpu())
