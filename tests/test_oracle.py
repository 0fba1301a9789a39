"""The CPU oracle against the golden vectors and the reference's known answers.

Parity pins for the restatement in oracle/ltxattn_oracle.c:
* MLXCapabilityTests.fusedAttention (Tests/LTXModulesTests/MLXCapabilityTests.swift:78-91)
* fixtures from an independent float64 torch implementation (tests/golden/make_golden.py)
* analytic known answers (uniform attention, one-hot keys, zero-angle RoPE, LSE)
"""
import hashlib
import json
import os

import numpy as np
import pytest

import oracle
from ltxattn import inputs


def sha(*arrays) -> str:
    """Same digest as tests/golden/make_golden.py records."""
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a, dtype=np.float32).tobytes())
    return h.hexdigest()


def load(golden_dir, name):
    z = np.load(os.path.join(golden_dir, name + ".npz"))
    meta = json.loads(str(z["meta"]))
    return meta, z


def regen(meta):
    s, B, H, Lq, Lk, D = meta["seed"], meta["B"], meta["H"], meta["Lq"], meta["Lk"], meta["D"]
    bf16, rms = meta["bf16"], meta["rmsnorm"]
    q = inputs.seeded_tensor(s + 2, (B, H, Lq, D), rmsnorm=rms, bf16=bf16)
    k = inputs.seeded_tensor(s + 3, (B, H, Lk, D), rmsnorm=rms, bf16=bf16)
    v = inputs.seeded_tensor(s + 4, (B, H, Lk, D), bf16=bf16)
    dout = inputs.seeded_tensor(s + 5, (B, H, Lq, D), bf16=bf16) if meta["grad"] else None
    return q, k, v, dout


def test_reference_known_answer_fused_attention():
    # MLXCapabilityTests.swift:80-90: q = k = 1, v = 2, H=4, T=16, D=64 -> 2.0 within 1e-4
    q = np.ones((1, 4, 16, 64), np.float32)
    v = np.full((1, 4, 16, 64), 2.0, np.float32)
    out, _ = oracle.attn_fwd(q, q, v)
    assert out.shape == (1, 4, 16, 64)
    assert abs(out[0, 0, 0, 0] - 2.0) < 1e-4
    assert np.all(np.abs(out - 2.0) < 1e-6)


@pytest.mark.parametrize("name", ["c1_fp32_256", "mask_cross_bf16", "mask_cross_fp32",
                                  "rope_self_bf16_d128", "rope_cross_bf16_d64",
                                  "grad_mask_fp32", "grad_rope_fp32"])
def test_oracle_matches_golden(golden_dir, name):
    meta, z = load(golden_dir, name)
    q, k, v, dout = regen(meta)
    assert sha(q, k, v, *([dout] if dout is not None else [])) == meta["input_sha256"]
    mask = z["mask"] if "mask" in z.files else None
    qt = (z["q_cos"], z["q_sin"]) if "q_cos" in z.files else None
    kt = (z["k_cos"], z["k_sin"]) if "k_cos" in z.files else None
    qr, kr = q, k
    if qt is not None:
        ktab = kt if kt is not None else qt
        qr = oracle.rope(q, qt[0], qt[1], meta["bf16"])
        kr = oracle.rope(k, ktab[0], ktab[1], meta["bf16"])
        tol = 0.0 if meta["bf16"] else 1e-6
        np.testing.assert_allclose(qr, z["q_rotated"], atol=tol, rtol=0)
        np.testing.assert_allclose(kr, z["k_rotated"], atol=tol, rtol=0)
    out, lse = oracle.attn_fwd(qr, kr, v, mask=mask)
    np.testing.assert_allclose(out, z["out"], atol=1e-6, rtol=0)
    np.testing.assert_allclose(lse, z["lse"], atol=1e-5, rtol=0)
    if meta["grad"]:
        dq, dk, dv = oracle.attn_bwd(qr, kr, v, dout, mask=mask)
        if qt is not None:
            ktab = kt if kt is not None else qt
            dq = oracle.rope_bwd(dq, qt[0], qt[1], False)
            dk = oracle.rope_bwd(dk, ktab[0], ktab[1], False)
        np.testing.assert_allclose(dq, z["dq"], atol=1e-5, rtol=0)
        np.testing.assert_allclose(dk, z["dk"], atol=1e-5, rtol=0)
        np.testing.assert_allclose(dv, z["dv"], atol=1e-5, rtol=0)


def test_generators_agree():
    # the package's numpy stream and the oracle's C stream are the same function
    a = inputs.normal(77, 100000)
    b = oracle.fill_normal(77, 100000)
    assert np.max(np.abs(a - b)) <= 1e-6 * np.max(np.abs(a))
    assert np.array_equal(inputs.round_bf16(a), oracle.round_bf16(a))


def test_bench_bits_is_the_reference_operand_stream():
    # Sources/ltx/Bench.swift:479-493 stepped one element at a time with Python
    # integers, against the vectorised restatement the benchmark uses
    mask = (1 << 64) - 1
    seed = 0x5EED + 2
    state = (seed + 0x9E3779B97F4A7C15) & mask
    want = []
    for _ in range(64):
        state = (state + 0x9E3779B97F4A7C15) & mask
        z = state
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & mask
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & mask
        z ^= z >> 31
        unit = np.float32(z >> 40) / np.float32(1 << 24)
        want.append((unit - np.float32(0.5)) * np.float32(2))
    got = inputs.bench_bits(seed, 64)
    assert np.array_equal(got, inputs.round_bf16(np.array(want, np.float32)))
    assert got.min() >= -1.0 and got.max() <= 1.0


def test_head_slices_are_slices_of_the_whole_tensor():
    whole = inputs.seeded_tensor(5, (2, 6, 10, 16), rmsnorm=True)
    part = inputs.seeded_tensor(5, (2, 6, 10, 16), rmsnorm=True, heads=(2, 3))
    assert np.array_equal(whole[:, 2:5], part)


def test_uniform_attention_is_mean_of_v():
    rng = np.random.default_rng(0)
    q = np.zeros((1, 2, 5, 64), np.float32)
    k = rng.standard_normal((1, 2, 9, 64)).astype(np.float32)
    v = rng.standard_normal((1, 2, 9, 64)).astype(np.float32)
    out, lse = oracle.attn_fwd(q, k, v)
    np.testing.assert_allclose(out, np.broadcast_to(v.mean(axis=2, keepdims=True), out.shape), atol=1e-6)
    np.testing.assert_allclose(lse, np.log(9.0), atol=1e-6)


def test_one_hot_key_and_mask_all_but_one():
    rng = np.random.default_rng(1)
    q = np.ones((1, 1, 3, 64), np.float32)
    k = np.zeros((1, 1, 7, 64), np.float32)
    k[0, 0, 4] = 10.0  # logit 80 against 0
    v = rng.standard_normal((1, 1, 7, 64)).astype(np.float32)
    out, _ = oracle.attn_fwd(q, k, v)
    np.testing.assert_allclose(out[0, 0], np.broadcast_to(v[0, 0, 4], (3, 64)), atol=1e-6)
    m = np.zeros((1, 7), np.uint8)
    m[0, 2] = 1
    out, _ = oracle.attn_fwd(q, np.ones_like(k), v, mask=m)
    np.testing.assert_allclose(out[0, 0], np.broadcast_to(v[0, 0, 2], (3, 64)), atol=1e-6)


def test_fully_masked_rows_are_unmasked():
    rng = np.random.default_rng(2)
    q = rng.standard_normal((1, 2, 4, 64)).astype(np.float32)
    k = rng.standard_normal((1, 2, 6, 64)).astype(np.float32)
    v = rng.standard_normal((1, 2, 6, 64)).astype(np.float32)
    a, la = oracle.attn_fwd(q, k, v, mask=np.zeros((1, 6), np.uint8))
    b, lb = oracle.attn_fwd(q, k, v)
    assert np.isfinite(a).all()
    np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(la, lb)


def test_rope_zero_angle_is_identity_and_relative():
    x = inputs.seeded_tensor(5, (1, 2, 8, 64), bf16=True)
    cos, sin = inputs.rope1d(np.zeros(8), 64)
    np.testing.assert_array_equal(oracle.rope(x, cos, sin, True), x)
    # relative-position invariance of q.k under a 1-D table (fp32, no rounding)
    c, s = inputs.rope1d(np.arange(8, dtype=np.float64), 64, bf16=False)
    q = np.broadcast_to(x[:, :, :1], x.shape).copy()
    qr = oracle.rope(q, c, s, False)
    dots = np.einsum("bhid,bhjd->bhij", qr, qr)
    for d in range(1, 4):
        diag = np.array([dots[0, 0, i, i + d] for i in range(8 - d)])
        np.testing.assert_allclose(diag, diag[0], rtol=1e-4, atol=1e-4)


def test_f32_mode_matches_f64_mode():
    q = inputs.seeded_tensor(11, (1, 2, 70, 64), bf16=False)
    k = inputs.seeded_tensor(12, (1, 2, 90, 64), bf16=False)
    v = inputs.seeded_tensor(13, (1, 2, 90, 64), bf16=False)
    m = np.ones((1, 90), np.uint8)
    m[0, 50:] = 0
    a, la = oracle.attn_fwd(q, k, v, mask=m)
    b, lb = oracle.attn_fwd_f32(q, k, v, mask=m)
    np.testing.assert_allclose(a, b, atol=2e-6)
    np.testing.assert_allclose(la, lb, atol=2e-5)


def test_backward_matches_finite_differences():
    rng = np.random.default_rng(3)
    q = rng.standard_normal((1, 1, 5, 8)).astype(np.float32)
    k = rng.standard_normal((1, 1, 6, 8)).astype(np.float32)
    v = rng.standard_normal((1, 1, 6, 8)).astype(np.float32)
    do = rng.standard_normal((1, 1, 5, 8)).astype(np.float32)
    dq, dk, dv = oracle.attn_bwd(q, k, v, do, scale=0.5)

    def loss(qq, kk, vv):
        o, _ = oracle.attn_fwd(qq, kk, vv, scale=0.5)
        return float(np.sum(o.astype(np.float64) * do))

    eps = 1e-2
    for arr, g in ((q, dq), (k, dk), (v, dv)):
        for idx in [(0, 0, 1, 3), (0, 0, 4, 0)]:
            p = arr.copy(); p[idx] += eps
            m = arr.copy(); m[idx] -= eps
            args_p = [p if arr is x else x for x in (q, k, v)]
            args_m = [m if arr is x else x for x in (q, k, v)]
            fd = (loss(*args_p) - loss(*args_m)) / (2 * eps)
            assert abs(fd - g[idx]) < 2e-3, (idx, fd, g[idx])


def test_streaming_key_backward_matches_the_full_backward():
    # oracle_attn_bwd_keys (rows streamed, lse and delta from a forward) against
    # oracle_attn_bwd on the same head, for a scattered set of keys
    q = inputs.seeded_tensor(21, (1, 1, 300, 64), rmsnorm=True)
    k = inputs.seeded_tensor(22, (1, 1, 257, 64), rmsnorm=True)
    v = inputs.seeded_tensor(23, (1, 1, 257, 64))
    do = inputs.seeded_tensor(24, (1, 1, 300, 64))
    dq, dk, dv = oracle.attn_bwd(q, k, v, do)
    out, lse = oracle.attn_fwd(q, k, v)
    delta = np.sum(out.astype(np.float64) * do, axis=-1)
    keys = [0, 1, 77, 128, 200, 256]
    dk_s, dv_s = oracle.attn_bwd_keys(q[0, 0], k[0, 0], v[0, 0], do[0, 0], lse[0, 0], delta[0, 0], keys)
    np.testing.assert_allclose(dk_s, dk[0, 0, keys], atol=2e-6)
    np.testing.assert_allclose(dv_s, dv[0, 0, keys], atol=2e-6)


def test_rotary_tables_c_restatement_matches_the_numpy_one():
    # DiTForward.rotary restated twice (C oracle, numpy helper): identical angle
    # arithmetic; the two fp32 cos/sin implementations differ by at most 2 ulp
    for pos, max_pos, inner, heads in ((inputs.video_positions(3, 4, 5), [20, 2048, 2048], 4096, 32),
                                       (inputs.audio_positions(40), [20], 2048, 32)):
        c, s = oracle.rotary_tables(pos, max_pos, inner, heads)
        rc, rs = inputs.reference_rotary(pos, inner, max_pos, heads, bf16=False)
        for a, b in ((c, rc), (s, rs)):
            assert a.shape == b.shape
            tol = 2 * np.spacing(np.abs(b).astype(np.float32))
            assert (np.abs(a.astype(np.float64) - b) <= tol).all()


def test_qk_prep_restatement():
    # rmsNorm over the inner dim (mean square, r = 1/sqrt(mean + eps), y = T(w * T(x * r)))
    # then the head split: the C oracle against the same formula in numpy
    x = inputs.seeded_tensor(5, (2, 9, 512), bf16=True) * 2.0
    w = inputs.round_bf16(np.random.default_rng(0).uniform(0.5, 1.5, 512).astype(np.float32))
    got = oracle.qk_prep(x, w, 4, 1e-6)
    ms = (x.astype(np.float64) ** 2).mean(-1, keepdims=True).astype(np.float32).astype(np.float64)
    r = (1.0 / np.sqrt(ms + np.float64(np.float32(1e-6)))).astype(np.float32)
    y = inputs.round_bf16(w * inputs.round_bf16(x * r))
    np.testing.assert_array_equal(got, y.reshape(2, 9, 4, 128).transpose(0, 2, 1, 3))


def test_gate_restatement_known_answers():
    # DiTAttention.swift:395-399: gates = 2 * sigmoid(logits), sigmoid in fp32 cast to bf16
    logits = np.array([[[0.0, 100.0, -100.0, 1.0]]], np.float32)  # [B=1, T=1, H=4]
    g = oracle.gate_value(logits, bf16=True)
    assert g[0, 0, 0] == 1.0 and g[0, 0, 1] == 2.0 and g[0, 0, 2] == 0.0
    s1 = 1.0 / (1.0 + np.exp(-1.0))
    assert g[0, 0, 3] == 2.0 * inputs.round_bf16(np.float32(s1))
    out = np.full((1, 4, 1, 8), 0.75, np.float32)  # [B, H, T, D]
    y = oracle.gate_output(out, logits, bf16=True)
    np.testing.assert_array_equal(y[0, :, 0, 0], inputs.round_bf16(0.75 * g[0, 0]))
    # fp32 activations: no rounding of the sigmoid
    assert oracle.gate_value(logits[..., 3:], bf16=False)[0, 0, 0] == np.float32(2.0 * np.float32(s1))


def test_module_composition_is_the_reference_order():
    # the oracle's whole module on a tiny case against the steps written out in
    # numpy: projections (matmul then bias, each rounded), rmsNorm + split + RoPE,
    # SDPA, gate, merge, to_out (DiTAttention.swift:315-404)
    rng = np.random.default_rng(1)
    B, T, heads, D = 1, 8, 4, 128
    dim = heads * D

    def bf(a):
        return inputs.round_bf16(np.asarray(a, np.float32))

    w = {n: bf(rng.normal(0, 1 / np.sqrt(dim), (dim, dim))) for n in ("to_q.weight", "to_k.weight",
                                                                       "to_v.weight", "to_out.0.weight")}
    w.update({n: bf(rng.uniform(-0.1, 0.1, dim)) for n in ("to_q.bias", "to_k.bias", "to_v.bias", "to_out.0.bias")})
    w.update({"q_norm.weight": bf(np.ones(dim)), "k_norm.weight": bf(np.ones(dim)),
              "to_gate_logits.weight": bf(rng.normal(0, 0.05, (heads, dim)))})
    x = bf(rng.normal(0, 1, (B, T, dim)))
    got = oracle.dit_attention_module(x, w, heads)

    def lin(a, n):
        y = bf(a.astype(np.float64) @ w[n + ".weight"].astype(np.float64).T)
        return bf(y.astype(np.float64) + w[n + ".bias"]) if n + ".bias" in w else y

    q = oracle.qk_prep(lin(x, "to_q"), w["q_norm.weight"], heads, 1e-6)
    k = oracle.qk_prep(lin(x, "to_k"), w["k_norm.weight"], heads, 1e-6)
    v = np.ascontiguousarray(lin(x, "to_v").reshape(B, T, heads, D).transpose(0, 2, 1, 3))
    att = bf(oracle.attn_fwd(q, k, v)[0])
    gated = oracle.gate_output(att, lin(x, "to_gate_logits"), True)
    want = lin(np.ascontiguousarray(gated.transpose(0, 2, 1, 3).reshape(B, T, dim)), "to_out.0")
    np.testing.assert_array_equal(got, want)
