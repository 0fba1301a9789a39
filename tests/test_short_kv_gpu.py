"""The persistent forward for key/value sequences of one 128-key tile
(fwd_short_sm100.cu; the audio->video cross-attention's 126 audio keys).

It runs when the planner chooses (num_splits 0, kv_len <= 128, more units than
SMs); num_splits=1 forces the one-CTA-per-unit forward kernel.  The two compute
each row with the same arithmetic, so their outputs and LSEs must agree bit
for bit; both are also checked against the CPU oracle (bf16 bar: max abs <=
2e-2, rel-L2 <= 1e-2).
"""
import numpy as np
import pytest
import torch

import oracle
from ltxattn import AttentionBackend, Rotary, device_info, device_status, inputs

pytestmark = pytest.mark.gpu
LSE_ABS = 2e-3


def dev(x, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dtype)


@pytest.fixture(autouse=True)
def no_kernel_timeouts():
    yield
    assert device_status(clear=True) == 0, "a kernel wait timed out"


def make(seed, B, H, Hk, Lq, Lk, D):
    q = inputs.seeded_tensor(seed + 2, (B, H, Lq, D), rmsnorm=True, bf16=True)
    k = inputs.seeded_tensor(seed + 3, (B, Hk, Lk, D), rmsnorm=True, bf16=True)
    v = inputs.seeded_tensor(seed + 4, (B, Hk, Lk, D), bf16=True)
    return q, k, v


def check(got, ref, what):
    g = got.float().cpu().numpy().astype(np.float64)
    err = np.abs(g - ref)
    rel = np.linalg.norm(err) / max(np.linalg.norm(ref), 1e-30)
    assert err.max() <= 2e-2 and rel <= 1e-2, f"{what}: max abs {err.max():.3e} rel-L2 {rel:.3e}"


def same_bits(a, b):
    return torch.equal(a.contiguous().view(torch.int16), b.contiguous().view(torch.int16))


def test_persistent_kernel_is_chosen_only_when_it_applies():
    sms = device_info()["sm_count"]
    q = torch.zeros((1, sms + 1, 256, 64), device="cuda", dtype=torch.bfloat16)
    kv = torch.zeros((1, sms + 1, 126, 64), device="cuda", dtype=torch.bfloat16)
    # no scratch: neither split partials nor rotated copies
    assert AttentionBackend.prepare(q, kv, kv).workspace is None


@pytest.mark.parametrize("D,Lk", [(64, 126), (128, 128), (64, 1), (128, 77)])
def test_matches_the_forward_kernel_bit_for_bit(D, Lk):
    # the audio->video shape: 3120 video queries per head, 32 heads
    B, H, Lq = 1, 32, 3120
    q, k, v = make(101 + D + Lk, B, H, H, Lq, Lk, D)
    qd, kd, vd = dev(q), dev(k), dev(v)
    out, lse = AttentionBackend.attention(qd, kd, vd, save_lse=True)
    one, lse1 = AttentionBackend.attention(qd, kd, vd, save_lse=True, num_splits=1)
    assert same_bits(out, one)
    assert torch.equal(lse, lse1)
    hs = [0, 7, 31]
    ref, ref_lse = oracle.attn_fwd(q[:, hs], k[:, hs], v[:, hs])
    check(out[:, hs], ref, f"D={D} Lk={Lk}")
    assert np.abs(lse[:, hs].cpu().numpy() - ref_lse).max() < LSE_ABS


@pytest.mark.parametrize("D", [64, 128])
def test_kv_reloads_inside_a_cta(D):
    # two query blocks per head: every CTA's range of units crosses heads and
    # batches, so K/V are reloaded mid-range behind units still using them
    B, H, Lq, Lk = 2, 160, 300, 100
    q, k, v = make(141 + D, B, H, H, Lq, Lk, D)
    qd, kd, vd = dev(q), dev(k), dev(v)
    out, lse = AttentionBackend.attention(qd, kd, vd, save_lse=True)
    one, lse1 = AttentionBackend.attention(qd, kd, vd, save_lse=True, num_splits=1)
    assert same_bits(out, one) and torch.equal(lse, lse1)
    hs = [0, 1, 2, 159]
    ref, _ = oracle.attn_fwd(q[:, hs], k[:, hs], v[:, hs])
    check(out[:, hs], ref, f"reloads D={D}")


def test_key_masks_and_the_free_row_rule():
    # batch 0: ragged mask; batch 1: no valid key -> every key (GemmaTextEncoder.swift:306-319)
    B, H, Lq, Lk, D = 2, 80, 300, 100, 128
    q, k, v = make(131, B, H, H, Lq, Lk, D)
    m = np.zeros((B, Lk), np.uint8)
    m[0] = np.random.default_rng(4).random(Lk) < 0.4
    md = torch.from_numpy(m).cuda()
    qd, kd, vd = dev(q), dev(k), dev(v)
    out, lse = AttentionBackend.attention(qd, kd, vd, key_mask=md, save_lse=True)
    one, lse1 = AttentionBackend.attention(qd, kd, vd, key_mask=md, save_lse=True, num_splits=1)
    assert same_bits(out, one) and torch.equal(lse, lse1)
    hs = [0, 41, 79]
    ref, _ = oracle.attn_fwd(q[:, hs], k[:, hs], v[:, hs], mask=m)
    check(out[:, hs], ref, "masked")


def test_rotary_gate_merged_view_and_grouped_heads():
    B, H, Hk, Lq, Lk, D = 1, 8, 2, 5000, 126, 64  # 20 query blocks x 8 heads = 160 units
    q, k, v = make(151, B, H, Hk, Lq, Lk, D)
    qd, kd, vd = dev(q), dev(k), dev(v)
    gate = dev(2.0 * inputs.seeded_tensor(157, (B, Lq, H)))
    merged = torch.empty((B, Lq, H * D), device="cuda", dtype=torch.bfloat16)
    view = merged.view(B, Lq, H, D).permute(0, 2, 1, 3)
    AttentionBackend.attention(qd, kd, vd, gate=gate, out=view)
    one, _ = AttentionBackend.attention(qd, kd, vd, gate=gate, num_splits=1)
    assert same_bits(view, one)
    # rotary tables (separate query and key clocks, the cross-modal case)
    H2 = 32
    q2, k2, v2 = make(161, 1, H2, H2, 3120, 126, 64)
    qc, qs = inputs.rope1d(inputs.video_frame_seconds(13, 240), 64)
    kc, ks = inputs.rope1d(inputs.audio_token_seconds(126), 64)
    rq, rk = Rotary(dev(qc), dev(qs)), Rotary(dev(kc), dev(ks))
    a, _ = AttentionBackend.attention(dev(q2), dev(k2), dev(v2), q_rotary=rq, k_rotary=rk)
    b, _ = AttentionBackend.attention(dev(q2), dev(k2), dev(v2), q_rotary=rq, k_rotary=rk, num_splits=1)
    assert same_bits(a, b)
    ref, _ = oracle.attention_reference(q2[:, :2], k2[:, :2], v2[:, :2], q_rot=(qc, qs), k_rot=(kc, ks), bf16=True)
    check(a[:, :2], ref, "cross-modal rotary")


def test_head_block_and_per_batch_masks():
    # a rank's head block of a sharded job, three batch rows with different masks
    # (one with no valid key), through the persistent kernel
    B, H, Lq, Lk, D = 3, 64, 640, 96, 128  # 3 query blocks x 56 heads x 3 batches = 504 units
    q, k, v = make(171, B, H, H, Lq, Lk, D)
    m = np.zeros((B, Lk), np.uint8)
    m[0, :50] = 1
    m[1] = np.random.default_rng(8).random(Lk) < 0.7
    md = torch.from_numpy(m).cuda()
    qd, kd, vd = dev(q), dev(k), dev(v)
    out = torch.zeros_like(qd)
    lse = torch.zeros((B, H, Lq), device="cuda", dtype=torch.float32)
    AttentionBackend.attention(qd, kd, vd, key_mask=md, out=out, lse=lse, head_begin=8, head_count=56)
    one = torch.zeros_like(qd)
    lse1 = torch.zeros_like(lse)
    AttentionBackend.attention(qd, kd, vd, key_mask=md, out=one, lse=lse1, head_begin=8, head_count=56, num_splits=1)
    assert same_bits(out, one) and torch.equal(lse, lse1)
    assert torch.count_nonzero(out[:, :8]).item() == 0  # heads outside the block untouched
    hs = [8, 40, 63]
    ref, ref_lse = oracle.attn_fwd(q[:, hs], k[:, hs], v[:, hs], mask=m)
    check(out[:, hs], ref, "head block")
    assert np.abs(lse[:, hs].cpu().numpy() - ref_lse).max() < LSE_ABS
