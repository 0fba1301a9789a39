"""ltxattn_allgather_heads through the C ABI on one GPU (a one-rank NCCL
communicator: the gather is then a copy with the documented layout)."""
import ctypes

import pytest
import torch

from ltxattn import _lib
from ltxattn.dist import HeadGather

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
