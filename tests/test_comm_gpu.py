"""ltxattn_allgather_heads through the C ABI on one GPU (a one-rank NCCL
communicator: the gather is then a copy with the documented layout)."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from ltxattn import _lib, inputs
from ltxattn.dist import HeadGather
from ltxattn.proj import linear

pytestmark = pytest.mark.gpu


def test_single_rank_gather_is_identity_layout():
    raw = (ctypes.c_uint8 * 128)()
    assert _lib.load().ltxattn_comm_unique_id(raw) == _lib.OK, _lib.last_error()
    g = HeadGather(1, 0, bytes(raw), torch.cuda.current_device())
    try:
        assert g.size() == (1, 0)  # what NCCL itself reports
        for dt in (torch.bfloat16, torch.float32):
            local = torch.randn(2, 4, 33, 64, device="cuda").to(dt)
            out = g.gather(local)
            torch.cuda.synchronize()
            assert out.shape == local.shape and torch.equal(out, local)
    finally:
        g.close()


def test_single_rank_row_parallel_to_out_is_the_plain_linear():
    # ltxattn_out_project_allreduce on a one-rank communicator: the fp32 partial, the
    # (identity) all-reduce and the bias / rounding pass give the bits of ltxattn_linear
    # without K splitting (the same single fp32 sum per output)
    raw = (ctypes.c_uint8 * 128)()
    assert _lib.load().ltxattn_comm_unique_id(raw) == _lib.OK, _lib.last_error()
    g = HeadGather(1, 0, bytes(raw), torch.cuda.current_device())
    try:
        m, n, k = 300, 512, 1024
        x = torch.from_numpy(inputs.seeded_tensor(61, (m, k))).to("cuda", torch.bfloat16)
        w = torch.from_numpy(inputs.round_bf16(inputs.seeded_tensor(62, (n, k)) / np.float32(32))).to(
            "cuda", torch.bfloat16)
        b = torch.from_numpy(inputs.round_bf16(inputs.seeded_tensor(63, (n,)) * np.float32(0.1))).to(
            "cuda", torch.bfloat16)
        got = g.out_project(x, w, b)
        want = linear(x, w, b, split_k=False)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
        ref = oracle.linear(x.float().cpu().numpy(), w.float().cpu().numpy(), b.float().cpu().numpy())
        err = np.abs(got.float().cpu().numpy() - ref)
        assert err.max() <= 2e-2 and np.linalg.norm(err) / np.linalg.norm(ref) <= 1e-2
        # a column block of a wider weight (the row-parallel layout: stride = the full k)
        wide = torch.zeros((n, 2 * k), device="cuda", dtype=torch.bfloat16)
        wide[:, k:] = w
        got2 = g.out_project(x, wide[:, k:], b)
        torch.cuda.synchronize()
        assert torch.equal(got2, want)
    finally:
        g.close()
