"""The attention module's projections on tcgen05, through the C ABI, against the
CPU oracle.

* ltxattn_linear (DiTAttention.linear, DiTAttention.swift:178-188): the fp64
  matmul rounded to bf16, plus the bias rounded again (oracle.linear); also
  against the library GEMM (cuBLAS through torch) with the same two roundings.
* ltxattn_qk_project / _pair (the q / k path :341-342,358-367 in one kernel):
  against oracle.qk_prep(oracle.linear(x)) and against the unfused composition
  (library GEMM + ltxattn_qk_prep).

Tolerances (bf16): max abs <= 2e-2 and rel-L2 <= 1e-2
against the oracle.  The fused and unfused paths may differ in the last bit of
the matmul (fp32 accumulation order), so they are compared in the same terms.
"""
import numpy as np
import pytest
import torch

import oracle
from ltxattn import Rotary, device_status, inputs, qk_prep
from ltxattn.proj import linear, qk_project, qk_project_pair

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


def _tables(T, D, H, per_head, seed):
    ang = np.arange(T, dtype=np.float64)[:, None] * (10000.0 ** (-np.arange(D // 2) / (D // 2)))[None, :]
    if per_head:
        ang = ang[None] * (1.0 + 0.01 * np.arange(H))[:, None, None]
        ang = ang[None]
    else:
        ang = ang[None, None]
    c = inputs.round_bf16(np.cos(ang).astype(np.float32))
    s = inputs.round_bf16(np.sin(ang).astype(np.float32))
    return c, s


@pytest.mark.parametrize("B,T,heads,D,k,rope,per_head,with_bias", [
    (1, 300, 32, 128, 4096, True, False, True),   # video: cluster of 8
    (1, 3120, 32, 128, 4096, True, False, True),  # config 2's q at full size
    (2, 200, 32, 64, 2048, True, True, True),     # audio: cluster of 4, per-head tables, batch 2
    (1, 129, 8, 64, 512, False, False, False),    # cluster of 1, no rotary, no bias
    (1, 64, 16, 128, 1024, True, True, False),
])
def test_qk_project_matches_the_oracle(B, T, heads, D, k, rope, per_head, with_bias):
    n = heads * D
    x = inputs.seeded_tensor(40 + T, (B, T, k))
    w = weights(41, n, k)
    b = bias(42, n) if with_bias else None
    nw = inputs.round_bf16(0.5 + inputs.seeded_tensor(43, (n,)) ** 2 * np.float32(0.25))
    c = s = None
    rot = None
    if rope:
        c, s = _tables(T, D, heads, per_head, 44)
        rot = Rotary(dev(c), dev(s))
    got = qk_project(dev(x), dev(w), dev(b) if b is not None else None, dev(nw), heads, rot)
    torch.cuda.synchronize()
    y = oracle.linear(x.reshape(B * T, k), w, b).reshape(B, T, n)
    ref = oracle.qk_prep(y, nw, heads, 1e-6, c, s, bf16=True)
    err = check(got, ref, f"qk_project B{B} T{T} {heads}x{D}")
    assert np.mean(err == 0) > 0.95
    # the unfused composition on the device: library GEMM, then ltxattn_qk_prep
    yd = (dev(x) @ dev(w).t())
    if b is not None:
        yd = yd + dev(b)
    unfused = qk_prep(yd, dev(nw), heads, rot)
    diff = (got.float() - unfused.float()).abs()
    assert diff.max().item() <= 2e-2 and (diff == 0).float().mean().item() > 0.95


def test_qk_project_pair_is_two_single_calls():
    # a cross-attention's q (300 query tokens) and k (1024 context tokens) in one launch
    heads, D, k = 32, 128, 4096
    n = heads * D
    xq = dev(inputs.seeded_tensor(50, (1, 300, k)))
    xk = dev(inputs.seeded_tensor(51, (1, 1024, k)))
    wq, wk = dev(weights(52, n, k)), dev(weights(53, n, k))
    bq, bk = dev(bias(54, n)), dev(bias(55, n))
    nq = dev(inputs.round_bf16(0.5 + inputs.seeded_tensor(56, (n,)) ** 2 * np.float32(0.25)))
    nk = dev(inputs.round_bf16(0.5 + inputs.seeded_tensor(57, (n,)) ** 2 * np.float32(0.25)))
    cq, sq = _tables(300, D, heads, False, 0)
    ck, sk = _tables(1024, D, heads, False, 0)
    rq, rk = Rotary(dev(cq), dev(sq)), Rotary(dev(ck), dev(sk))
    pq, pk = qk_project_pair(xq, wq, bq, nq, xk, wk, bk, nk, heads, rq, rk)
    oq = qk_project(xq, wq, bq, nq, heads, rq)
    ok = qk_project(xk, wk, bk, nk, heads, rk)
    torch.cuda.synchronize()
    assert torch.equal(pq, oq) and torch.equal(pk, ok)
    # deterministic: a second pair call gives the same bits
    pq2, pk2 = qk_project_pair(xq, wq, bq, nq, xk, wk, bk, nk, heads, rq, rk)
    assert torch.equal(pq, pq2) and torch.equal(pk, pk2)
