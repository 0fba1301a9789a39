"""Rotary tables on a B200 (``ltxattn_rotary_tables``, DiTForward.rotary at
DiTForward.swift:641-678) against the C oracle's restatement.

The angle arithmetic is the same sequence of separately rounded fp32 ops on
both sides; cos and sin come from CUDA's and the host libm's accurate fp32
functions, which may differ by an ulp or two.  Tolerances: fp32 tables within
4 ulp of the oracle; bf16 tables (the oracle's fp32 rounded to bf16) within one
bf16 ulp, differing in under 1% of entries.
"""
import numpy as np
import pytest
import torch

import oracle
from ltxattn import Failure, inputs, rotary_tables

pytestmark = pytest.mark.gpu

CASES = {
    # video self-attn: inner 4096 -> 682 freqs x 3 dims + 2 identity pairs, 64 per head
    "video_3120": (lambda: inputs.video_positions(13, 12, 20), [20, 2048, 2048], 4096, 32),
    # audio: inner 2048, one dimension, 32 per head
    "audio_126": (lambda: inputs.audio_positions(126), [20], 2048, 32),
}


@pytest.mark.parametrize("case", sorted(CASES))
def test_fp32_tables_match_the_oracle(case):
    make_pos, max_pos, inner, heads = CASES[case]
    pos = make_pos()
    want_c, want_s = oracle.rotary_tables(pos, max_pos, inner, heads)
    rot = rotary_tables(torch.from_numpy(pos).cuda(), max_pos, inner, heads, dtype=torch.float32)
    torch.cuda.synchronize()
    for got, want in ((rot.cos, want_c), (rot.sin, want_s)):
        g = got.cpu().numpy()
        assert g.shape == want.shape
        tol = 4 * np.spacing(np.abs(want).astype(np.float32)) + 1e-30
        bad = np.abs(g.astype(np.float64) - want.astype(np.float64)) > tol
        assert not bad.any(), f"{case}: {bad.sum()} entries beyond 4 ulp"


@pytest.mark.parametrize("case", sorted(CASES))
def test_bf16_tables_are_the_fp32_tables_narrowed(case):
    make_pos, max_pos, inner, heads = CASES[case]
    pos = make_pos()
    want_c, want_s = oracle.rotary_tables(pos, max_pos, inner, heads)
    rot = rotary_tables(torch.from_numpy(pos).cuda(), max_pos, inner, heads, dtype=torch.bfloat16)
    torch.cuda.synchronize()
    for got, want in ((rot.cos, want_c), (rot.sin, want_s)):
        g = got.float().cpu().numpy().astype(np.float64)
        w = inputs.round_bf16(want).astype(np.float64)
        ulp = np.spacing(np.abs(w).astype(np.float32)).astype(np.float64) * 65536.0  # bf16 ulp
        assert (np.abs(g - w) <= ulp + 1e-30).all(), case
        assert (g != w).mean() < 0.01, case


def test_identity_pad_and_head_split():
    # video 4096: the first two rotary pairs of head 0 are the leading identity pad
    pos = inputs.video_positions(2, 3, 4)
    rot = rotary_tables(torch.from_numpy(pos).cuda(), [20, 2048, 2048], 4096, 32, dtype=torch.float32)
    c, s = rot.cos.cpu().numpy(), rot.sin.cpu().numpy()
    assert c.shape == (1, 32, 24, 64)
    assert (c[0, 0, :, :2] == 1.0).all() and (s[0, 0, :, :2] == 0.0).all()
    assert not (c[0, 1, :, :2] == 1.0).all()


def test_argument_errors_are_refused():
    pos = torch.zeros((3, 4, 2), device="cuda")
    with pytest.raises(Failure):
        rotary_tables(pos, [20, 2048, 2048], 4096, 30)  # 2048 pairs do not split into 30 heads
    with pytest.raises(Failure):
        rotary_tables(pos, [0, 2048, 2048], 4096, 32)  # zero normaliser
