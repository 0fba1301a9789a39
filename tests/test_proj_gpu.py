"""The attention module's projections on tcgen05, through the C ABI, against the
CPU oracle.

* ltxattn_linear (DiTAttention.linear, DiTAttention.swift:178-188): the fp64
  matmul rounded to bf16, plus the bias rounded again (oracle.linear); also
  against the library GEMM (cuBLAS through torch) with the same two roundings.

Tolerances (bf16): max abs <= 2e-2 and rel-L2 <= 1e-2
against the oracle; the fp32-accumulated GEMM and the oracle's fp64 sum round
to the same bf16 in almost every entry (asserted).
"""
import numpy as np
import pytest
import torch

import oracle
from ltxattn import device_status, inputs
from ltxattn.proj import linear

pytestmark = pytest.mark.gpu


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda", torch.bfloat16)


def host(t):
    return t.float().cpu().numpy()


def check(got, ref, what):
    g = host(got) if isinstance(got, torch.Tensor) else got
    err = np.abs(g.astype(np.float64) - ref.astype(np.float64))
    rel = float(np.linalg.norm(err) / max(np.linalg.norm(ref), 1e-30))
    assert err.max() <= 2e-2 and rel <= 1e-2, f"{what}: max abs {err.max():.3e} rel-L2 {rel:.3e}"
    return err


@pytest.fixture(autouse=True)
def no_kernel_timeouts():
    yield
    assert device_status(clear=True) == 0, "a kernel wait timed out"


def weights(seed, n, k, scale=None):
    w = inputs.seeded_tensor(seed, (n, k), bf16=True) * np.float32(scale if scale else 1.0 / np.sqrt(k))
    return inputs.round_bf16(w)


def bias(seed, n):
    return inputs.round_bf16(inputs.seeded_tensor(seed, (n,)) * np.float32(0.1))


@pytest.mark.parametrize("m,n,k,with_bias", [
    (300, 256, 512, True),      # ragged rows, one column tile
    (200, 2048, 2048, True),    # audio projection width
    (129, 4096, 4096, False),   # video width, one row past a tile
    (3120, 32, 4096, True),     # to_gate_logits: [3120, 4096] -> 32 heads
    (96, 128, 256, True),
    (64, 64, 64, True),
    (100, 8, 512, True),        # eight heads' gate logits: a ragged 32-column tile
    (130, 296, 256, True),      # 256 + a ragged tile of 40
])
def test_linear_matches_the_oracle(m, n, k, with_bias):
    x = inputs.seeded_tensor(10 + m, (m, k))
    w = weights(20 + n, n, k)
    b = bias(30 + n, n) if with_bias else None
    got = linear(dev(x), dev(w), dev(b) if b is not None else None)
    torch.cuda.synchronize()
    ref = oracle.linear(x, w, b)
    err = check(got, ref, f"linear {m}x{n}x{k}")
    # the oracle's fp64 sum and the kernel's fp32 sum round to the same bf16 almost everywhere
    assert np.mean(err == 0) > 0.97


def test_linear_full_size_against_the_library_gemm():
    # config 2's to_q: [3120, 4096] x [4096, 4096]^T + b, against cuBLAS (torch) with the
    # reference's two roundings
    m, n, k = 3120, 4096, 4096
    x = dev(inputs.seeded_tensor(3, (m, k)))
    w = dev(weights(4, n, k))
    b = dev(bias(5, n))
    got = linear(x, w, b)
    want = (x @ w.t()) + b
    torch.cuda.synchronize()
    diff = (got.float() - want.float()).abs()
    assert diff.max().item() <= 2e-2
    assert (diff == 0).float().mean().item() > 0.97
    # and the oracle on a sample of rows
    rows = np.r_[0:64, 1500:1564, 3056:3120]
    ref = oracle.linear(host(x)[rows], host(w), host(b))
    check(got[torch.as_tensor(rows, device="cuda")], ref, "linear full size (rows)")


def test_linear_views_and_batches():
    # a [B, T, k] input with a padded row stride, and an output view into a wider buffer
    B, T, k, n = 2, 150, 512, 256
    base = dev(inputs.seeded_tensor(7, (B, T, k + 64)))
    x = base[:, :, :k]
    w = dev(weights(8, n, k))
    wide = torch.zeros((B * T, n + 32), device="cuda", dtype=torch.bfloat16)
    for bi in range(B):
        o = linear(x[bi], w, out=wide[bi * T:(bi + 1) * T, :n])
        ref = oracle.linear(host(x[bi]), host(w))
        check(o, ref, f"strided batch {bi}")
    assert torch.all(wide[:, n:] == 0)  # nothing written past the view


@pytest.mark.parametrize("m,n,k", [(3120, 32, 4096), (300, 8, 2048), (200, 64, 1024)])
def test_split_k_for_narrow_outputs(m, n, k):
    # narrow outputs split K across CTAs (fp32 partials added in a fixed order,
    # then the bias and the roundings): against the oracle, against the unsplit
    # kernel, and bit-identical on a second call
    x = inputs.seeded_tensor(70 + n, (m, k))
    w = weights(71 + n, n, k)
    b = bias(72 + n, n)
    got = linear(dev(x), dev(w), dev(b))
    again = linear(dev(x), dev(w), dev(b))
    unsplit = linear(dev(x), dev(w), dev(b), split_k=False)
    torch.cuda.synchronize()
    err = check(got, oracle.linear(x, w, b), f"split-K linear {m}x{n}x{k}")
    assert np.mean(err == 0) > 0.97
    assert torch.equal(got, again)
    # the two fp32 summation orders round the product to the same bf16 almost
    # everywhere, else one ulp of the product apart; the bias is added after that
    # rounding, so the tolerance scales with |product| <= |out| + |bias| (two ulps
    # of that bound also cover the final rounding)
    diff = (got.float() - unsplit.float()).abs()
    ulp = (unsplit.float().abs() + dev(b).float().abs()) * 2.0 ** -6
    assert bool(torch.all(diff <= ulp)) and (diff == 0).float().mean().item() > 0.97
