"""q / k preparation on a B200 (``ltxattn_qk_prep``: rmsNorm over the inner
dim, head split, split RoPE -- DiTAttention.swift:358-367) against the CPU oracle.

The device reduces the mean square in an fp32 tree, the oracle in fp64; the
normaliser r can differ in its last ulp, which moves a bf16 rounding only for
values within an ulp of a rounding midpoint.  Tolerance: bf16 outputs within
2 bf16 ulps of the oracle and equal in > 99% of entries; fp32 outputs within
a relative 1e-5 of the oracle.
"""
import numpy as np
import pytest
import torch

import oracle
from ltxattn import Failure, Rotary, inputs, qk_prep

pytestmark = pytest.mark.gpu


def norm_weight(inner, seed=3, bf16=True):
    w = np.random.default_rng(seed).uniform(0.5, 1.5, inner).astype(np.float32)
    return inputs.round_bf16(w) if bf16 else w


def compare(got, want, dtype, what):
    g = got.float().cpu().numpy().astype(np.float64)
    w = want.astype(np.float64)
    if dtype == torch.bfloat16:
        ulp = np.spacing(np.abs(want).astype(np.float32)).astype(np.float64) * 65536.0
        assert (np.abs(g - w) <= 2 * ulp + 1e-30).all(), what
        assert (g != w).mean() < 0.01, what
    else:
        assert np.abs(g - w).max() <= 1e-5 * max(1.0, np.abs(w).max()), what


@pytest.mark.parametrize("dtype,H,D,tables", [(torch.bfloat16, 32, 128, "per_head"),
                                              (torch.bfloat16, 32, 128, "shared"),
                                              (torch.bfloat16, 32, 64, "none"),
                                              (torch.float32, 32, 64, "per_head")])
def test_qk_prep_matches_oracle(dtype, H, D, tables):
    B, T, inner = 2, 150, H * D
    bf = dtype == torch.bfloat16
    x = inputs.seeded_tensor(8, (B, T, inner), bf16=bf) * 3.0
    if bf:
        x = inputs.round_bf16(x)  # the device sees bf16 values: give the oracle the same ones
    w = norm_weight(inner, bf16=bf)
    cos = sin = None
    if tables == "per_head":
        n_pos = 3 if D == 128 else 1
        pos = inputs.video_positions(3, 5, 10) if n_pos == 3 else inputs.audio_positions(T)
        mp = [20, 2048, 2048] if n_pos == 3 else [20]
        cos, sin = inputs.reference_rotary(pos, inner, mp, H, bf16=bf)
    elif tables == "shared":
        cos, sin = inputs.rope1d(np.arange(T, dtype=np.float64), D, bf16=bf)
    want = oracle.qk_prep(x, w, H, 1e-6, cos, sin, bf16=bf)
    rot = None if cos is None else Rotary(torch.from_numpy(cos).to("cuda", dtype), torch.from_numpy(sin).to("cuda", dtype))
    got = qk_prep(torch.from_numpy(x).to("cuda", dtype), torch.from_numpy(w).to("cuda", dtype), H, rot, eps=1e-6)
    torch.cuda.synchronize()
    compare(got, want, dtype, f"{dtype} H{H} D{D} {tables}")


def test_qk_prep_reads_a_fused_projection_row_and_writes_a_strided_view():
    # x is the q third of a [B, T, 3 * inner] fused projection; out is a [B, T, H, D]
    # buffer seen as [B, H, T, D] (the reference's transposed split view)
    dtype, B, T, H, D = torch.bfloat16, 1, 64, 32, 128
    inner = H * D
    qkv = inputs.seeded_tensor(9, (B, T, 3 * inner), bf16=True)
    w = norm_weight(inner)
    cos, sin = inputs.rope1d(np.arange(T, dtype=np.float64), D)
    want = oracle.qk_prep(np.ascontiguousarray(qkv[:, :, :inner]), w, H, 1e-6, cos, sin)
    xd = torch.from_numpy(qkv).to("cuda", dtype)[:, :, :inner]
    buf = torch.empty((B, T, H, D), device="cuda", dtype=dtype)
    rot = Rotary(torch.from_numpy(cos).to("cuda", dtype), torch.from_numpy(sin).to("cuda", dtype))
    qk_prep(xd, torch.from_numpy(w).to("cuda", dtype), H, rot, out=buf.permute(0, 2, 1, 3))
    torch.cuda.synchronize()
    compare(buf.permute(0, 2, 1, 3), want, dtype, "strided")


def test_qk_prep_refuses_unsupported_widths():
    x = torch.zeros((1, 4, 24 * 16), device="cuda", dtype=torch.bfloat16)  # inner 384
    with pytest.raises(Failure):
        qk_prep(x, torch.ones(384, device="cuda", dtype=torch.bfloat16), 6)


@pytest.mark.parametrize("dtype,Tq,Tk,D", [(torch.bfloat16, 150, 150, 128), (torch.bfloat16, 300, 126, 64),
                                           (torch.float32, 40, 70, 64)])
def test_pair_matches_two_single_calls(dtype, Tq, Tk, D):
    # ltxattn_qk_prep_pair: q and k (token counts may differ) in one launch, the same bits
    from ltxattn import qk_prep_pair
    H, B = 32, 2
    inner = H * D
    bf = dtype == torch.bfloat16
    xq = torch.from_numpy(inputs.seeded_tensor(21, (B, Tq, inner), bf16=bf) * 2.0).to("cuda", dtype)
    xk = torch.from_numpy(inputs.seeded_tensor(22, (B, Tk, inner), bf16=bf) * 2.0).to("cuda", dtype)
    wq = torch.from_numpy(norm_weight(inner, 4, bf)).to("cuda", dtype)
    wk = torch.from_numpy(norm_weight(inner, 5, bf)).to("cuda", dtype)
    cq, sq = inputs.rope1d(np.arange(Tq, dtype=np.float64), D, bf16=bf)
    ck, sk = inputs.rope1d(np.arange(Tk, dtype=np.float64) * 0.5, D, bf16=bf)
    rq = Rotary(torch.from_numpy(cq).to("cuda", dtype), torch.from_numpy(sq).to("cuda", dtype))
    rk = Rotary(torch.from_numpy(ck).to("cuda", dtype), torch.from_numpy(sk).to("cuda", dtype))
    qh, kh = qk_prep_pair(xq, wq, xk, wk, H, rq, rk)
    q1 = qk_prep(xq, wq, H, rq)
    k1 = qk_prep(xk, wk, H, rk)
    torch.cuda.synchronize()
    # (the single calls are checked against the oracle above)
    assert torch.equal(qh, q1) and torch.equal(kh, k1)


def test_pair_with_a_strided_input_takes_two_launches():
    # an x view whose rows are not 16-byte aligned cannot stream by bulk copies:
    # the pair falls back to two single launches, with the same results
    from ltxattn import qk_prep_pair
    H, D, T = 32, 64, 20
    inner = H * D
    base = torch.from_numpy(inputs.seeded_tensor(23, (1, T, inner + 1))).to("cuda", torch.bfloat16)
    xq = base[:, :, 1:]  # offset by one element
    xk = torch.from_numpy(inputs.seeded_tensor(24, (1, T, inner))).to("cuda", torch.bfloat16)
    w = torch.from_numpy(norm_weight(inner)).to("cuda", torch.bfloat16)
    qh, kh = qk_prep_pair(xq, w, xk, w, H)
    torch.cuda.synchronize()
    assert torch.equal(qh, qk_prep(xq, w, H)) and torch.equal(kh, qk_prep(xk, w, H))
