"""Backward parity on a B200: dQ, dK, dV through the C ABI against the CPU
oracle's closed-form VJP (fp64 accumulation) on the same seeded inputs.

The reference pins no attention gradient (its only backward fixture is a
single linear layer, TrainingBackwardGateTests.swift:28-34), so the oracle's
VJP is itself pinned by finite differences and by torch-autograd golden
vectors (tests/test_oracle.py).  Tolerances: float32 max abs <= 1e-5 (scaled
by the gradient's magnitude); bf16 max abs <= 2e-2 relative to the largest
gradient entry and rel-L2 <= 1e-2.
"""
import json
import os

import numpy as np
import pytest
import torch

import oracle
from ltxattn import AttentionBackend, Rotary, device_status, inputs

pytestmark = pytest.mark.gpu


def dev(x, dtype):
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dtype)


def check_grad(got, ref, dtype, what, reduce_len=128):
    """Gradient tolerance.

    float32: max abs <= 1e-5 * max(1, |ref|_inf) * sqrt(max(1, reduce_len / 128)) -- the
    north star's 1e-5, widened by the square root of how many fp32 terms each gradient
    entry sums beyond one 128-wide tile (cancellation in dP - Delta is fp32 noise).
    bf16: max abs <= 2e-2 * max(1, |ref|_inf) and rel-L2 <= 1e-2, the rel-L2 denominator
    floored at 1e-3 per element so an all-zero exact gradient (one key: P == 1, dS == 0)
    is judged by its absolute error.
    """
    g = got.float().cpu().numpy().astype(np.float64)
    r = ref.astype(np.float64)
    err = np.abs(g - r)
    scale = max(1.0, float(np.abs(r).max()))
    if dtype == torch.float32:
        tol = 1e-5 * scale * np.sqrt(max(1.0, reduce_len / 128.0))
        assert err.max() <= tol, f"{what} max abs {err.max():.3e} (tol {tol:.2e})"
    else:
        denom = max(np.linalg.norm(r), 1e-3 * np.sqrt(r.size))
        rel = float(np.linalg.norm(err) / denom)
        assert err.max() <= 2e-2 * scale and rel <= 1e-2, f"{what} max abs {err.max():.3e} rel-L2 {rel:.3e}"


@pytest.fixture(autouse=True)
def no_kernel_timeouts():
    yield
    assert device_status(clear=True) == 0, "a kernel wait timed out"


def run_case(B, H, Lq, Lk, D, dtype, seed, mask=None, q_tab=None, k_tab=None, rmsnorm=True):
    bf = dtype == torch.bfloat16
    q = inputs.seeded_tensor(seed + 2, (B, H, Lq, D), rmsnorm=rmsnorm, bf16=bf)
    k = inputs.seeded_tensor(seed + 3, (B, H, Lk, D), rmsnorm=rmsnorm, bf16=bf)
    v = inputs.seeded_tensor(seed + 4, (B, H, Lk, D), bf16=bf)
    do = inputs.seeded_tensor(seed + 5, (B, H, Lq, D), bf16=bf)
    qd, kd, vd, dod = dev(q, dtype), dev(k, dtype), dev(v, dtype), dev(do, dtype)
    md = torch.from_numpy(mask).cuda() if mask is not None else None
    qr = Rotary(dev(q_tab[0], dtype), dev(q_tab[1], dtype)) if q_tab is not None else None
    kr = Rotary(dev(k_tab[0], dtype), dev(k_tab[1], dtype)) if k_tab is not None else None
    out, lse = AttentionBackend.attention(qd, kd, vd, key_mask=md, q_rotary=qr, k_rotary=kr, save_lse=True)
    dq, dk, dv = AttentionBackend.attention_backward(qd, kd, vd, out, dod, lse, key_mask=md, q_rotary=qr,
                                                     k_rotary=kr)
    # oracle: rotate (bf16 arithmetic as the reference), VJP, then transpose rotation
    qo, ko = q, k
    if q_tab is not None:
        kt = k_tab if k_tab is not None else q_tab
        qo = oracle.rope(q, q_tab[0], q_tab[1], bf)
        ko = oracle.rope(k, kt[0], kt[1], bf)
    rq, rk, rv = oracle.attn_bwd(qo, ko, v, do, mask=mask)
    if q_tab is not None:
        rq = oracle.rope_bwd(rq, q_tab[0], q_tab[1], bf)
        rk = oracle.rope_bwd(rk, kt[0], kt[1], bf)
    return (dq, dk, dv), (rq, rk, rv)


SHAPES = [
    (1, 2, 128, 128, 128),
    (1, 2, 200, 333, 128),
    (2, 2, 130, 70, 64),
    (1, 3, 1, 257, 64),
    (1, 2, 300, 1, 128),
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", SHAPES)
def test_backward_matches_oracle(shape, dtype):
    got, ref = run_case(*shape, dtype, seed=100 + shape[2])
    Lq, Lk = shape[2], shape[3]
    for name, g, r, n in zip(("dq", "dk", "dv"), got, ref, (Lk, Lq, Lq)):
        check_grad(g, r, dtype, f"{name} {shape}", reduce_len=n)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_backward_masked(dtype):
    B, H, Lq, Lk, D = 3, 2, 150, 400, 64
    m = np.zeros((B, Lk), np.uint8)
    m[0, :94] = 1
    m[1] = np.random.default_rng(3).random(Lk) < 0.4
    # batch 2 fully masked -> un-masked attention
    got, ref = run_case(B, H, Lq, Lk, D, dtype, seed=300, mask=m)
    for name, g, r, n in zip(("dq", "dk", "dv"), got, ref, (Lk, Lq, Lq)):
        check_grad(g, r, dtype, f"{name} masked", reduce_len=n)
    # masked keys receive exactly zero gradient
    dk, dv = got[1].float().cpu().numpy(), got[2].float().cpu().numpy()
    assert np.all(dk[0, :, 94:] == 0) and np.all(dv[0, :, 94:] == 0)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_backward_with_rope(dtype):
    bf = dtype == torch.bfloat16
    H, D = 4, 128
    T = 3 * 4 * 10
    tab = inputs.reference_rotary(inputs.video_positions(3, 4, 10), inner=H * D, max_pos=[20, 2048, 2048],
                                  heads=H, bf16=bf)
    got, ref = run_case(1, H, T, T, D, dtype, seed=400, q_tab=tab)
    for name, g, r in zip(("dq", "dk", "dv"), got, ref):
        check_grad(g, r, dtype, f"{name} rope")


def test_backward_cross_modal_tables():
    dtype = torch.bfloat16
    H, D, Lq, Lk = 4, 64, 13 * 12, 126
    qt = inputs.rope1d(inputs.video_frame_seconds(13, 12), D)
    kt = inputs.rope1d(inputs.audio_token_seconds(Lk), D)
    got, ref = run_case(1, H, Lq, Lk, D, dtype, seed=500, q_tab=qt, k_tab=kt)
    for name, g, r in zip(("dq", "dk", "dv"), got, ref):
        check_grad(g, r, dtype, f"{name} cross rope")


@pytest.mark.parametrize("name", ["grad_mask_fp32", "grad_rope_fp32"])
def test_backward_golden(golden_dir, name):
    z = np.load(os.path.join(golden_dir, name + ".npz"))
    meta = json.loads(str(z["meta"]))
    mask = z["mask"] if "mask" in z.files else None
    tab = (z["q_cos"], z["q_sin"]) if "q_cos" in z.files else None
    got, _ = run_case(meta["B"], meta["H"], meta["Lq"], meta["Lk"], meta["D"], torch.float32, meta["seed"],
                      mask=mask, q_tab=tab, rmsnorm=meta["rmsnorm"])
    for g, key in zip(got, ("dq", "dk", "dv")):
        check_grad(g, z[key], torch.float32, f"{name} {key}")


def test_backward_deterministic_and_head_range():
    B, H, T, D = 1, 6, 700, 128
    dtype = torch.bfloat16
    q = dev(inputs.seeded_tensor(602, (B, H, T, D), rmsnorm=True), dtype)
    k = dev(inputs.seeded_tensor(603, (B, H, T, D), rmsnorm=True), dtype)
    v = dev(inputs.seeded_tensor(604, (B, H, T, D)), dtype)
    do = dev(inputs.seeded_tensor(605, (B, H, T, D)), dtype)
    out, lse = AttentionBackend.attention(q, k, v, save_lse=True)
    a = AttentionBackend.attention_backward(q, k, v, out, do, lse)
    b = AttentionBackend.attention_backward(q, k, v, out, do, lse)
    for x, y in zip(a, b):
        assert torch.equal(x, y)  # gradient checkpointing recomputes: bit-identical
    part = [torch.full_like(t, 5.0) for t in a]
    AttentionBackend.attention_backward(q, k, v, out, do, lse, head_begin=2, head_count=3, dq=part[0], dk=part[1],
                                        dv=part[2])
    for x, y in zip(a, part):
        assert torch.equal(x[:, 2:5], y[:, 2:5])
        assert torch.all(y[:, :2] == 5.0) and torch.all(y[:, 5:] == 5.0)


def test_backward_large_shape_subset():
    # config 5's shape is 29760 tokens; a 2-head slice at 3120 tokens keeps the
    # oracle in seconds while exercising many tiles in both directions.
    got, ref = run_case(1, 2, 3120, 3120, 128, torch.bfloat16, seed=700)  # bf16: no length widening
    for name, g, r in zip(("dq", "dk", "dv"), got, ref):
        check_grad(g, r, torch.bfloat16, f"{name} 3120")
