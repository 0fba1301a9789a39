"""Split RoPE on a B200 (``ltxattn_rope``, the device code ``ltxattn_fwd`` also
uses to rotate q and k) against the CPU oracle, bit for bit.

The reference op is ``applySplitRoPE`` (DiTAttention.swift:206-234): in bf16
every product and every sum rounds to bf16; in fp32 the four products and two
sums are plain unfused fp32 operations.  Both are integer-exact comparisons
here: the bf16 bits (or fp32 bits) must equal the oracle's.
"""
import numpy as np
import pytest
import torch

import oracle
from ltxattn import Rotary, apply_split_rope, inputs

pytestmark = pytest.mark.gpu


def bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).cpu().numpy()
    return t.contiguous().view(torch.int32).cpu().numpy()


def oracle_bits(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, dtype) -> np.ndarray:
    y = oracle.rope(x, cos, sin, bf16=dtype == torch.bfloat16)
    return bits(torch.from_numpy(y).to(dtype))


def wide_values(rng, shape, lo=-40, hi=40):
    """bf16-exact values with random signs, 8-bit significands and exponents in
    [lo, hi]: products and sums of these reach every rounding case, including
    operands far apart in magnitude."""
    sig = 1.0 + rng.integers(0, 128, size=shape) / 128.0
    e = rng.integers(lo, hi + 1, size=shape).astype(np.float64)
    sgn = np.where(rng.random(shape) < 0.5, -1.0, 1.0)
    return (sgn * sig * np.exp2(e)).astype(np.float32)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("tables", ["grid3d", "per_head_random"])
def test_rope_bit_exact(dtype, D, tables):
    B, H, T = 2, 3, 97
    bf = dtype == torch.bfloat16
    x = inputs.seeded_tensor(11, (B, H, T, D), rmsnorm=True, bf16=bf)
    if tables == "grid3d":
        cos, sin = inputs.rope3d_grid(1, 8, 13, D, bf16=bf)  # [1, 1, 104, D/2]
        cos, sin = cos[:, :, :T], sin[:, :, :T]
    else:
        rng = np.random.default_rng(5)
        ang = rng.uniform(-20, 20, size=(1, H, T, D // 2))
        cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
        if bf:
            cos, sin = inputs.round_bf16(cos), inputs.round_bf16(sin)
    xd = torch.from_numpy(x).to("cuda", dtype)
    rot = Rotary(torch.from_numpy(np.ascontiguousarray(cos)).to("cuda", dtype),
                 torch.from_numpy(np.ascontiguousarray(sin)).to("cuda", dtype))
    out = apply_split_rope(xd, rot)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bits(out), oracle_bits(x, cos, sin, dtype))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_rope_bit_exact_wide_magnitudes(dtype):
    # operands 2^-40 .. 2^40 in x and in the tables: sums of terms far apart in
    # magnitude and products near rounding midpoints, over 1.6 M rotary pairs
    rng = np.random.default_rng(7)
    B, H, T, D = 1, 4, 3200, 128
    x = wide_values(rng, (B, H, T, D))
    cos = wide_values(rng, (1, H, T, D // 2), -20, 20)
    sin = wide_values(rng, (1, H, T, D // 2), -20, 20)
    if dtype == torch.bfloat16:
        x, cos, sin = inputs.round_bf16(x), inputs.round_bf16(cos), inputs.round_bf16(sin)
    xd = torch.from_numpy(x).to("cuda", dtype)
    rot = Rotary(torch.from_numpy(cos).to("cuda", dtype), torch.from_numpy(sin).to("cuda", dtype))
    out = apply_split_rope(xd, rot)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bits(out), oracle_bits(x, cos, sin, dtype))


def test_rope_strided_unaligned_and_in_place_views():
    # the transposed split view of the reference (a [B, T, H, D] buffer seen as
    # [B, H, T, D]), a view whose start is not 16-byte aligned (element path),
    # and rotation in place must all give the oracle's bits
    dtype = torch.bfloat16
    B, H, T, D = 2, 4, 40, 64
    x = inputs.seeded_tensor(21, (B, H, T, D), rmsnorm=True, bf16=True)
    cos, sin = inputs.rope1d(np.arange(T, dtype=np.float64), D, bf16=True)
    want = oracle_bits(x, cos, sin, dtype)
    rot = Rotary(torch.from_numpy(cos).to("cuda", dtype), torch.from_numpy(sin).to("cuda", dtype))

    bthd = torch.from_numpy(np.ascontiguousarray(x.transpose(0, 2, 1, 3))).to("cuda", dtype)
    view = bthd.permute(0, 2, 1, 3)  # [B, H, T, D] with strides (T*H*D, D, H*D, 1)
    np.testing.assert_array_equal(bits(apply_split_rope(view, rot)), want)

    flat = torch.empty(B * H * T * D + 1, device="cuda", dtype=dtype)
    odd = flat[1:].view(B, H, T, D)  # 2-byte offset: not 16-byte aligned
    odd.copy_(torch.from_numpy(x).to("cuda", dtype))
    np.testing.assert_array_equal(bits(apply_split_rope(odd, rot)), want)

    xd = torch.from_numpy(x).to("cuda", dtype)
    apply_split_rope(xd, rot, out=xd)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bits(xd), want)
