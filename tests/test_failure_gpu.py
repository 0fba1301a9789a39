"""Failure detection on the GPU, without a fault.

A kernel's bounded wait is made to run out on purpose: ltxattn_selftest_wait_timeout
launches one CTA that waits, with the attention kernels' own bounded wait, on
an mbarrier nothing ever arrives at, under a 1 ms limit.  The wait must give
up, record the timeout and its site in the device error word, free its tensor
memory and return; the host must read LTXATTN_ERR_TIMEOUT through
ltxattn_device_status; and the next ordinary call must run clean and correct
on the same context.  Nothing here traps, faults or hangs the GPU.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from ltxattn import AttentionBackend, _lib, device_status, inputs

pytestmark = pytest.mark.gpu

SELFTEST_SITE = 99


def _status():
    site = ctypes.c_int32(-1)
    rc = _lib.load().ltxattn_device_status(1, ctypes.byref(site))
    return rc, site.value


def test_a_wait_that_cannot_complete_times_out_and_the_context_stays_usable():
    assert device_status(clear=True) == 0
    L = _lib.load()
    stream = torch.cuda.current_stream()
    for _ in range(2):  # twice: the cleared word records the second timeout too
        rc = L.ltxattn_selftest_wait_timeout(1000, ctypes.c_void_p(stream.cuda_stream))
        assert rc == _lib.OK, _lib.last_error()
        torch.cuda.synchronize()  # the CTA gave up and exited
        rc, site = _status()
        assert rc == _lib.ERR_TIMEOUT and site == SELFTEST_SITE, (rc, site)
        assert "site 99" in _lib.last_error()
        assert device_status(clear=True) == 0  # read-and-clear left it clean

    # the next ordinary call on the same context: no error, oracle parity
    B, H, T, D = 1, 2, 300, 128
    q = inputs.seeded_tensor(52, (B, H, T, D), rmsnorm=True)
    k = inputs.seeded_tensor(53, (B, H, T, D), rmsnorm=True)
    v = inputs.seeded_tensor(54, (B, H, T, D))
    dev = lambda x: torch.from_numpy(x).to("cuda", torch.bfloat16)
    out, _ = AttentionBackend.attention(dev(q), dev(k), dev(v))
    torch.cuda.synchronize()
    assert device_status(clear=True) == 0
    ref, _ = oracle.attn_fwd(q, k, v)
    err = np.abs(out.float().cpu().numpy() - ref)
    assert err.max() <= 2e-2 and np.linalg.norm(err) / np.linalg.norm(ref) <= 1e-2


def test_the_timeout_is_reported_to_a_stream_it_was_not_launched_on():
    # the error word is per device, not per stream: a timeout on a side stream
    # is visible to the host after any device-wide synchronisation
    side = torch.cuda.Stream()
    rc = _lib.load().ltxattn_selftest_wait_timeout(2000, ctypes.c_void_p(side.cuda_stream))
    assert rc == _lib.OK
    rc, site = _status()  # ltxattn_device_status synchronises the device
    assert rc == _lib.ERR_TIMEOUT and site == SELFTEST_SITE
    assert device_status(clear=True) == 0
