"""The persistent forward over whole units (fwd_persist_sm100.cu): one CTA per
SM walks units c, c + G, c + 2G, ... and overlaps the end of one unit with the
start of the next.

The planner chooses it (ltxattn_fwd_plan kernel 3) for unbanded bf16 calls of at
least a wave of units when its cost model beats the one-CTA-per-unit kernel:
short KV ranges (the text cross-attention's one live tile of 1024 slots; fewer
than ~12 KV tiles at three rounds).  num_splits=1 forces the one-CTA-per-unit
kernel over whole units.  Both compute each unit with the same arithmetic, so
their outputs and LSEs must agree bit for bit; the persistent result is also
checked against the CPU oracle (bf16 bar: max abs <= 2e-2, rel-L2 <= 1e-2).
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from ltxattn import AttentionBackend, Rotary, _lib, device_info, device_status, inputs

pytestmark = pytest.mark.gpu
LSE_ABS = 2e-3


def dev(x, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dtype)


@pytest.fixture(autouse=True)
def no_kernel_timeouts():
    yield
    assert device_status(clear=True) == 0, "a kernel wait timed out"


def plan_kernel(B, H, Lq, Lk, D):
    a = _lib.FwdArgs()
    a.dtype, a.batch, a.heads, a.q_len, a.kv_len, a.head_dim = _lib.BF16, B, H, Lq, Lk, D
    info = _lib.FwdPlanInfo()
    assert _lib.load().ltxattn_fwd_plan(ctypes.byref(a), ctypes.byref(info)) == _lib.OK, _lib.last_error()
    return info.kernel


def same_bits(a, b):
    return torch.equal(a.contiguous().view(torch.int16), b.contiguous().view(torch.int16))


def check(got, ref, what):
    g = got.float().cpu().numpy().astype(np.float64)
    err = np.abs(g - ref)
    rel = np.linalg.norm(err) / max(np.linalg.norm(ref), 1e-30)
    assert err.max() <= 2e-2 and rel <= 1e-2, f"{what}: max abs {err.max():.3e} rel-L2 {rel:.3e}"


def test_video_queries_against_short_keys_match_bit_for_bit():
    # the video queries of config 2 (3120 tokens, 32 heads, 3D RoPE, the output
    # gate) against 1024 keys rotated by the first 1024 rows of the same table
    B, H, T, Lk, D = 1, 32, 3120, 1024, 128
    assert device_info()["sm_count"] == 148 and plan_kernel(B, H, T, Lk, D) == 3
    q = inputs.seeded_tensor(201, (B, H, T, D), rmsnorm=True)
    k = inputs.seeded_tensor(202, (B, H, Lk, D), rmsnorm=True)
    v = inputs.seeded_tensor(203, (B, H, Lk, D))
    gate = inputs.seeded_tensor(204, (B, T, H), bf16=True)
    cos, sin = inputs.rope3d_grid(13, 12, 20, D)
    rot = Rotary(dev(cos), dev(sin))
    qd, kd, vd, gd = dev(q), dev(k), dev(v), dev(gate)
    out, lse = AttentionBackend.attention(qd, kd, vd, q_rotary=rot, save_lse=True, gate=gd)
    one, lse1 = AttentionBackend.attention(qd, kd, vd, q_rotary=rot, save_lse=True, gate=gd, num_splits=1)
    assert same_bits(out, one)
    assert torch.equal(lse, lse1)
    # a second call on the same buffers: nothing carried over between calls
    again, _ = AttentionBackend.attention(qd, kd, vd, q_rotary=rot, save_lse=True, gate=gd)
    assert same_bits(again, out)
    hs = [0, 31]
    qr = oracle.round_bf16(oracle.rope(inputs.round_bf16(q[:, hs]), cos, sin, True))
    kr = oracle.round_bf16(oracle.rope(inputs.round_bf16(k[:, hs]), cos[:, :, :Lk], sin[:, :, :Lk], True))
    ref, ref_lse = oracle.attn_fwd(qr, kr, inputs.round_bf16(v[:, hs]))
    want = oracle.gate_output(oracle.round_bf16(ref), gate[:, :, hs], True)
    check(out[:, hs], want, "video queries, short keys")
    assert np.abs(lse[:, hs].cpu().numpy() - ref_lse).max() < LSE_ABS


@pytest.mark.parametrize("B,H,Lq,Lk,D", [
    (1, 150, 300, 500, 64),    # ragged query blocks (the second has no rows in Q tile 1), ragged last KV tile
    (2, 80, 400, 640, 128),    # two batches: units cross batches inside a CTA's walk
    (1, 40, 3120, 768, 64),    # D = 64 at the video length: 520 units, 3.5 per CTA
])
def test_mixed_units_match_bit_for_bit_and_the_oracle(B, H, Lq, Lk, D):
    assert plan_kernel(B, H, Lq, Lk, D) == 3
    q = inputs.seeded_tensor(211 + D, (B, H, Lq, D), rmsnorm=True, bf16=True)
    k = inputs.seeded_tensor(212 + D, (B, H, Lk, D), rmsnorm=True, bf16=True)
    v = inputs.seeded_tensor(213 + D, (B, H, Lk, D), bf16=True)
    qd, kd, vd = dev(q), dev(k), dev(v)
    out, lse = AttentionBackend.attention(qd, kd, vd, save_lse=True)
    one, lse1 = AttentionBackend.attention(qd, kd, vd, save_lse=True, num_splits=1)
    assert same_bits(out, one)
    assert torch.equal(lse, lse1)
    hs = [0, H // 2, H - 1]
    ref, ref_lse = oracle.attn_fwd(q[:, hs], k[:, hs], v[:, hs])
    check(out[:, hs], ref, f"B={B} H={H} Lq={Lq} Lk={Lk} D={D}")
    assert np.abs(lse[:, hs].cpu().numpy() - ref_lse).max() < LSE_ABS


def test_head_block_of_a_larger_tensor():
    # head_begin / head_count select heads 8..47 of 64: local head indexing of the
    # unit walk against global q / k / v / out coordinates
    B, H, Lq, Lk, D = 1, 64, 2304, 640, 128
    h0, hc = 8, 40
    assert plan_kernel(B, hc, Lq, Lk, D) == 3
    q = inputs.seeded_tensor(221, (B, H, Lq, D), rmsnorm=True, bf16=True)
    k = inputs.seeded_tensor(222, (B, H, Lk, D), rmsnorm=True, bf16=True)
    v = inputs.seeded_tensor(223, (B, H, Lk, D), bf16=True)
    qd, kd, vd = dev(q), dev(k), dev(v)
    out = torch.full((B, H, Lq, D), 7.0, device="cuda", dtype=torch.bfloat16)
    AttentionBackend.attention(qd, kd, vd, head_begin=h0, head_count=hc, out=out)
    one = torch.full_like(out, 7.0)
    AttentionBackend.attention(qd, kd, vd, head_begin=h0, head_count=hc, out=one, num_splits=1)
    assert same_bits(out, one)
    assert torch.all(out[:, :h0] == 7.0) and torch.all(out[:, h0 + hc:] == 7.0)
    hs = [h0, h0 + hc - 1]
    ref, _ = oracle.attn_fwd(q[:, hs], k[:, hs], v[:, hs])
    check(out[:, hs], ref, "head block")


@pytest.mark.parametrize("B,H,Lq,Lk,D,valid", [
    (1, 32, 3120, 1024, 128, 94),   # config 3: text cross-attention, 94 of 1024 slots valid (one live tile)
    (2, 80, 600, 1000, 64, None),   # batch 0 a random mask, batch 1 no valid key (every key)
])
def test_key_masks_match_bit_for_bit_and_the_oracle(B, H, Lq, Lk, D, valid):
    assert device_info()["sm_count"] == 148
    q = inputs.seeded_tensor(231 + D, (B, H, Lq, D), rmsnorm=True, bf16=True)
    k = inputs.seeded_tensor(232 + D, (B, H, Lk, D), rmsnorm=True, bf16=True)
    v = inputs.seeded_tensor(233 + D, (B, H, Lk, D), bf16=True)
    m = np.zeros((B, Lk), np.uint8)
    if valid is not None:
        m[:, :valid] = 1
    else:
        m[0] = np.random.default_rng(5).random(Lk) < 0.3
    a = _lib.FwdArgs()
    a.dtype, a.batch, a.heads, a.q_len, a.kv_len, a.head_dim = _lib.BF16, B, H, Lq, Lk, D
    a.key_mask, a.key_mask_stride_b = 4096, Lk
    info = _lib.FwdPlanInfo()
    assert _lib.load().ltxattn_fwd_plan(ctypes.byref(a), ctypes.byref(info)) == _lib.OK
    assert info.kernel == 3
    qd, kd, vd, md = dev(q), dev(k), dev(v), torch.from_numpy(m).cuda()
    out, lse = AttentionBackend.attention(qd, kd, vd, key_mask=md, save_lse=True)
    one, lse1 = AttentionBackend.attention(qd, kd, vd, key_mask=md, save_lse=True, num_splits=1)
    assert same_bits(out, one)
    assert torch.equal(lse, lse1)
    hs = [0, H - 1]
    ref, ref_lse = oracle.attn_fwd(q[:, hs], k[:, hs], v[:, hs], mask=m)
    check(out[:, hs], ref, f"mask B={B} D={D}")
    assert np.abs(lse[:, hs].cpu().numpy() - ref_lse).max() < LSE_ABS
