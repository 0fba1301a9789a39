"""ltxattn_fwd_noalloc through the C ABI, against ltxattn_fwd.

Some callers cannot allocate device memory for the forward's scratch (a host
whose device memory belongs to another framework's allocator, or a render loop
that must not allocate between steps); ltxattn_fwd_noalloc serves them from a
fixed 32 MiB array inside the library.  This file runs last (pytest collects
files in name order) so that a failure here leaves every other test already
run; it also passes when run alone in a fresh process.

Each case is called twice, with a call of another shape and other data in
between: the shared array keeps the previous call's contents, so the second
call of a case starts from scratch bytes another call wrote and must not
depend on them.  Every case needs scratch (asserted), so the array is always
exercised; one case is also checked against the CPU oracle directly.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from ltxattn import AttentionBackend, Rotary, _lib, inputs

pytestmark = pytest.mark.gpu

BF16_MAX_ABS = 2e-2
BF16_REL_L2 = 1e-2


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda", torch.bfloat16)


def _case(B, H, Lq, Lk, D, seed, rope=False):
    q = _dev(inputs.seeded_tensor(seed + 2, (B, H, Lq, D), rmsnorm=True))
    k = _dev(inputs.seeded_tensor(seed + 3, (B, H, Lk, D), rmsnorm=True))
    v = _dev(inputs.seeded_tensor(seed + 4, (B, H, Lk, D)))
    qr = kr = None
    if rope:
        qc, qs = inputs.rope1d(np.arange(Lq, dtype=np.float64), D)
        kc, ks = inputs.rope1d(np.arange(Lk, dtype=np.float64) * 0.5, D)
        qr, kr = Rotary(_dev(qc), _dev(qs)), Rotary(_dev(kc), _dev(ks))
    return q, k, v, qr, kr


def _noalloc(q, k, v, qr, kr):
    out = torch.empty_like(q)
    lse = torch.empty(q.shape[:3], dtype=torch.float32, device=q.device)
    a, out = AttentionBackend.make_fwd_args(q, k, v, 1.0 / np.sqrt(q.shape[-1]), q_rotary=qr, k_rotary=kr,
                                            lse=lse, out=out)
    L = _lib.load()
    assert L.ltxattn_fwd_workspace(ctypes.byref(a)) > 0  # the case really uses the scratch array
    rc = L.ltxattn_fwd_noalloc(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == _lib.OK, _lib.last_error()
    torch.cuda.synchronize()
    return out, lse


def _check(got, ref):
    err = (got.float() - ref.float()).abs()
    rel = (err.norm() / ref.float().norm()).item()
    assert err.max().item() <= BF16_MAX_ABS and rel <= BF16_REL_L2, (err.max().item(), rel)


@pytest.mark.parametrize("shape,rope", [
    ((1, 8, 126, 3120, 64), True),     # short queries: split-KV partials live in the scratch
    ((1, 4, 300, 300, 128), True),     # rotated q / k copies live in the scratch
    ((2, 4, 200, 1000, 64), False),    # split-KV without rotary tables
])
def test_noalloc_matches_fwd_on_two_calls(shape, rope):
    B, H, Lq, Lk, D = shape
    q, k, v, qr, kr = _case(B, H, Lq, Lk, D, seed=900 + Lq, rope=rope)
    ref, ref_lse = AttentionBackend.attention(q, k, v, q_rotary=qr, k_rotary=kr, save_lse=True)
    # a call of another shape and other data, so the array holds other bytes
    other = _case(1, 6, 140, 2000, 128, seed=77, rope=True)
    for i in range(2):
        out, lse = _noalloc(q, k, v, qr, kr)
        _check(out, ref)
        assert (lse - ref_lse).abs().max().item() <= 2e-3
        if i == 0:
            _noalloc(*other)


def test_noalloc_against_the_oracle():
    B, H, Lq, Lk, D = 1, 4, 126, 3120, 64
    seed = 930
    qh = inputs.seeded_tensor(seed + 2, (B, H, Lq, D), rmsnorm=True)
    kh = inputs.seeded_tensor(seed + 3, (B, H, Lk, D), rmsnorm=True)
    vh = inputs.seeded_tensor(seed + 4, (B, H, Lk, D))
    out, lse = _noalloc(_dev(qh), _dev(kh), _dev(vh), None, None)
    ref, ref_lse = oracle.attn_fwd(qh, kh, vh)
    _check(out.cpu(), torch.from_numpy(ref))
    assert np.abs(lse.cpu().numpy() - ref_lse).max() <= 2e-3


def test_noalloc_refuses_scratch_beyond_its_array():
    B, H, Lq, Lk, D = 1, 64, 4096, 4096, 128  # rotated q and k copies alone need 128 MiB
    q, k, v, qr, kr = _case(1, 1, 8, 8, D, seed=1, rope=True)
    a = _lib.FwdArgs()
    a.dtype, a.batch, a.heads, a.q_len, a.kv_len, a.head_dim = _lib.BF16, B, H, Lq, Lk, D
    a.q_rotary = _lib.Rotary(qr.cos.data_ptr(), qr.sin.data_ptr(), 0, 0, D // 2, 1 << 20)
    a.k_rotary = _lib.Rotary(kr.cos.data_ptr(), kr.sin.data_ptr(), 0, 0, D // 2, 1 << 20)
    L = _lib.load()
    rc = L.ltxattn_fwd_noalloc(ctypes.byref(a), None)
    assert rc == _lib.ERR_WORKSPACE
    assert "ltxattn_fwd_noalloc" in _lib.last_error()
