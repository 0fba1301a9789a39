"""The per-head output gate fused into the forward's store (``gate`` of
``ltxattn_fwd_args``; DiTAttention.swift:395-404): out = T(T(O) * 2 *
T(sigmoid(logit))) per query row and head, against the CPU oracle and against
the un-gated kernel output gated on the host.

Tolerances: bf16 max abs <= 2e-2 and rel-L2 <= 1e-2 against the oracle; fp32
max abs <= 1e-5.  Against the un-gated output the gated one is the same bf16
product except where the device's fp32 sigmoid and the oracle's fp64 one round
to different bf16 values (a tie within one fp32 ulp): < 0.1% of entries.
"""
import numpy as np
import pytest
import torch

import oracle
from ltxattn import AttentionBackend, device_status, inputs

pytestmark = pytest.mark.gpu


def dev(x, dtype):
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dtype)


@pytest.fixture(autouse=True)
def no_kernel_timeouts():
    yield
    assert device_status(clear=True) == 0, "a kernel wait timed out"


def make(seed, B, H, Lq, Lk, D, bf):
    q = inputs.seeded_tensor(seed + 2, (B, H, Lq, D), rmsnorm=True, bf16=bf)
    k = inputs.seeded_tensor(seed + 3, (B, H, Lk, D), rmsnorm=True, bf16=bf)
    v = inputs.seeded_tensor(seed + 4, (B, H, Lk, D), bf16=bf)
    logits = 2.0 * inputs.seeded_tensor(seed + 6, (B, H, Lq), bf16=False)  # stored [B, H, T]
    if bf:
        logits = inputs.round_bf16(logits)
    return q, k, v, logits


@pytest.mark.parametrize("dtype,D,splits", [(torch.bfloat16, 128, 1), (torch.bfloat16, 64, 1),
                                            (torch.bfloat16, 128, 3), (torch.float32, 64, 0)])
def test_gate_matches_the_oracle(dtype, D, splits):
    bf = dtype == torch.bfloat16
    B, H, Lq, Lk = 2, 3, 300, 260
    q, k, v, logits = make(51 + D, B, H, Lq, Lk, D, bf)
    qd, kd, vd = dev(q, dtype), dev(k, dtype), dev(v, dtype)
    gate = dev(logits, dtype).transpose(1, 2)  # [B, T, H] view with strides (H*T, 1, T)
    out, _ = AttentionBackend.attention(qd, kd, vd, gate=gate, num_splits=splits)
    ref, _ = oracle.attn_fwd(q, k, v)
    want = oracle.gate_output(oracle.round_bf16(ref) if bf else ref, logits.transpose(0, 2, 1), bf)
    g = out.float().cpu().numpy()
    err = np.abs(g.astype(np.float64) - want)
    if bf:
        rel = np.linalg.norm(err) / np.linalg.norm(want)
        assert err.max() <= 2e-2 and rel <= 1e-2, (err.max(), rel)
        # the same product as gating the un-gated kernel output on the host
        plain, _ = AttentionBackend.attention(qd, kd, vd, num_splits=splits)
        host = oracle.gate_output(plain.float().cpu().numpy(), logits.transpose(0, 2, 1), True)
        assert (g != host).mean() < 1e-3
    else:
        assert err.max() <= 1e-5, err.max()


@pytest.mark.parametrize("splits", [1, 4])
def test_zero_logits_leave_the_output_unchanged(splits):
    # 2 * T(sigmoid(0)) = 1 exactly: the gated store equals the plain one bit for bit
    B, H, Lq, Lk, D = 1, 4, 256, 512, 128
    q, k, v, _ = make(61, B, H, Lq, Lk, D, True)
    qd, kd, vd = dev(q, torch.bfloat16), dev(k, torch.bfloat16), dev(v, torch.bfloat16)
    zero = torch.zeros((B, Lq, H), device="cuda", dtype=torch.bfloat16)
    gated, _ = AttentionBackend.attention(qd, kd, vd, gate=zero, num_splits=splits)
    plain, _ = AttentionBackend.attention(qd, kd, vd, num_splits=splits)
    assert torch.equal(gated.view(torch.int16), plain.view(torch.int16))


def test_closed_gates_zero_their_heads_and_the_merge_view():
    # a head whose logits are very negative is switched off; out is the merged
    # [B, T, H * D] buffer (DiTAttention.swift:401-403) seen as [B, H, T, D]
    B, H, Lq, Lk, D = 1, 4, 130, 130, 64
    q, k, v, _ = make(71, B, H, Lq, Lk, D, True)
    qd, kd, vd = dev(q, torch.bfloat16), dev(k, torch.bfloat16), dev(v, torch.bfloat16)
    logits = torch.zeros((B, Lq, H), device="cuda", dtype=torch.bfloat16)
    logits[:, :, 2] = -100.0
    merged = torch.empty((B, Lq, H * D), device="cuda", dtype=torch.bfloat16)
    view = merged.view(B, Lq, H, D).permute(0, 2, 1, 3)
    AttentionBackend.attention(qd, kd, vd, gate=logits, out=view)
    plain, _ = AttentionBackend.attention(qd, kd, vd)
    m = merged.view(B, Lq, H, D)
    assert torch.count_nonzero(m[:, :, 2]).item() == 0
    for h in (0, 1, 3):
        assert torch.equal(m[:, :, h].view(torch.int16), plain[:, h].view(torch.int16))
