"""Forward parity on a B200: the CUDA path (through the C ABI) against the CPU
oracle on the same seeded inputs.

Tolerances: float32 max abs error <= 1e-5; bfloat16 max
abs error <= 2e-2 and relative L2 error <= 1e-2, both against the fp64-
accumulated oracle on the same bf16-rounded inputs.
"""
import json
import os

import numpy as np
import pytest
import torch

import oracle
from ltxattn import AttentionBackend, Rotary, device_info, device_status, inputs, scaled_dot_product_attention

pytestmark = pytest.mark.gpu

F32_MAX_ABS = 1e-5
BF16_MAX_ABS = 2e-2
BF16_REL_L2 = 1e-2
LSE_ABS = 2e-3


def dev(x, dtype):
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dtype)


def check(got, ref, dtype, what=""):
    g = got.float().cpu().numpy() if isinstance(got, torch.Tensor) else got
    err = np.abs(g.astype(np.float64) - ref.astype(np.float64))
    max_abs = float(err.max()) if err.size else 0.0
    if dtype == torch.float32:
        assert max_abs <= F32_MAX_ABS, f"{what} max abs {max_abs:.3e}"
    else:
        rel = float(np.linalg.norm(err) / max(np.linalg.norm(ref), 1e-30))
        assert max_abs <= BF16_MAX_ABS and rel <= BF16_REL_L2, f"{what} max abs {max_abs:.3e} rel-L2 {rel:.3e}"


def make(seed, B, H, Lq, Lk, D, dtype, rms=True):
    bf = dtype == torch.bfloat16
    q = inputs.seeded_tensor(seed + 2, (B, H, Lq, D), rmsnorm=rms, bf16=bf)
    k = inputs.seeded_tensor(seed + 3, (B, H, Lk, D), rmsnorm=rms, bf16=bf)
    v = inputs.seeded_tensor(seed + 4, (B, H, Lk, D), bf16=bf)
    return q, k, v


@pytest.fixture(autouse=True)
def no_kernel_timeouts():
    yield
    assert device_status(clear=True) == 0, "a kernel wait timed out"


def test_reference_known_answer():
    # MLXCapabilityTests.swift:78-91: q = k = 1, v = 2, B1 H4 T16 D64 -> 2.0 within 1e-4
    for dt in (torch.float32, torch.bfloat16):
        q = torch.ones((1, 4, 16, 64), device="cuda", dtype=dt)
        v = torch.full((1, 4, 16, 64), 2.0, device="cuda", dtype=dt)
        out = scaled_dot_product_attention(q, q, v, scale=1.0 / 8.0)
        assert out.shape == (1, 4, 16, 64)
        assert abs(out[0, 0, 0, 0].item() - 2.0) < 1e-4
        assert torch.all((out.float() - 2.0).abs() < 1e-4)


def test_config1_fp32_against_golden(golden_dir):
    z = np.load(os.path.join(golden_dir, "c1_fp32_256.npz"))
    meta = json.loads(str(z["meta"]))
    q, k, v = make(meta["seed"], 1, 4, 256, 256, 64, torch.float32, rms=False)
    out, lse = AttentionBackend.attention(dev(q, torch.float32), dev(k, torch.float32), dev(v, torch.float32),
                                          1.0 / 8.0, save_lse=True)
    check(out, z["out"], torch.float32, "c1 vs golden")
    ref, ref_lse = oracle.attn_fwd(q, k, v)
    check(out, ref, torch.float32, "c1 vs oracle")
    assert np.abs(lse.cpu().numpy() - ref_lse).max() < 1e-5


SHAPES = [
    # B, H, Lq, Lk, D
    (1, 2, 128, 128, 128),
    (1, 2, 256, 384, 128),
    (2, 3, 17, 129, 64),
    (1, 4, 126, 126, 64),
    (1, 2, 1, 1, 64),
    (1, 2, 1, 300, 128),
    (1, 1, 300, 1000, 128),
    (2, 2, 385, 257, 64),
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", SHAPES)
def test_forward_matches_oracle(shape, dtype):
    B, H, Lq, Lk, D = shape
    q, k, v = make(7 + Lq + Lk, B, H, Lq, Lk, D, dtype)
    out, lse = AttentionBackend.attention(dev(q, dtype), dev(k, dtype), dev(v, dtype), save_lse=True)
    ref, ref_lse = oracle.attn_fwd(q, k, v)
    check(out, ref, dtype, f"{shape}")
    tol = 1e-5 if dtype == torch.float32 else LSE_ABS
    assert np.abs(lse.cpu().numpy() - ref_lse).max() < tol


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_key_padding_masks(dtype):
    B, H, Lq, Lk, D = 3, 2, 200, 1024, 128
    q, k, v = make(11, B, H, Lq, Lk, D, dtype)
    m = np.zeros((B, Lk), np.uint8)
    m[0, :94] = 1                 # config 3: first 94 of 1024 slots valid (one live KV tile)
    rng = np.random.default_rng(5)
    m[1] = rng.random(Lk) < 0.3   # ragged, every tile partial
    # batch 2: no valid key -> un-masked (GemmaTextEncoder.swift:306-319)
    out, lse = AttentionBackend.attention(dev(q, dtype), dev(k, dtype), dev(v, dtype),
                                          key_mask=torch.from_numpy(m).cuda(), save_lse=True)
    ref, ref_lse = oracle.attn_fwd(q, k, v, mask=m)
    check(out, ref, dtype, "masked")
    assert np.isfinite(out.float().cpu().numpy()).all()
    assert np.abs(lse.cpu().numpy() - ref_lse).max() < (1e-5 if dtype == torch.float32 else LSE_ABS)


def test_unaligned_mask_rows_give_the_same_result():
    # aligned rows take 16-byte loads, unaligned ones byte loads: same bits, same output
    B, H, Lq, Lk, D = 2, 2, 130, 300, 64
    q, k, v = make(29, B, H, Lq, Lk, D, torch.bfloat16)
    rng = np.random.default_rng(9)
    m = (rng.random((B, Lk)) < 0.5).astype(np.uint8)
    qd, kd, vd = dev(q, torch.bfloat16), dev(k, torch.bfloat16), dev(v, torch.bfloat16)
    aligned = torch.from_numpy(m).cuda()
    wide = torch.zeros((B, Lk + 1), dtype=torch.uint8, device="cuda")
    wide[:, 1:] = aligned
    odd = wide[:, 1:]  # base and row stride not 16-byte multiples
    a, _ = AttentionBackend.attention(qd, kd, vd, key_mask=aligned)
    b, _ = AttentionBackend.attention(qd, kd, vd, key_mask=odd)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    ref, _ = oracle.attn_fwd(q, k, v, mask=m)
    check(a, ref, torch.bfloat16, "aligned mask")


def test_mask_with_one_valid_key_returns_that_value_row():
    B, H, Lq, Lk, D = 1, 2, 64, 700, 64
    q, k, v = make(13, B, H, Lq, Lk, D, torch.bfloat16)
    m = np.zeros((1, Lk), np.uint8)
    m[0, 555] = 1
    out, _ = AttentionBackend.attention(dev(q, torch.bfloat16), dev(k, torch.bfloat16), dev(v, torch.bfloat16),
                                        key_mask=torch.from_numpy(m).cuda())
    want = np.broadcast_to(v[:, :, 555:556, :], out.shape)
    assert np.array_equal(out.float().cpu().numpy(), want)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("per_head", [False, True])
def test_rope_self_attention(dtype, per_head):
    bf = dtype == torch.bfloat16
    T, H, D = 3 * 4 * 5, 4, 128
    q, k, v = make(17, 1, H, T, T, D, dtype)
    if per_head:
        cos, sin = inputs.reference_rotary(inputs.video_positions(3, 4, 5), inner=H * D,
                                           max_pos=[20, 2048, 2048], heads=H, bf16=bf)
    else:
        cos, sin = inputs.rope3d_grid(3, 4, 5, D, bf16=bf)
    rot = Rotary(dev(cos, dtype), dev(sin, dtype))
    out, lse = AttentionBackend.attention(dev(q, dtype), dev(k, dtype), dev(v, dtype), q_rotary=rot, save_lse=True)
    ref, ref_lse = oracle.attention_reference(q, k, v, q_rot=(cos, sin), bf16=bf)
    check(out, ref, dtype, f"rope per_head={per_head}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_rope_cross_modal_separate_tables(dtype):
    bf = dtype == torch.bfloat16
    H, D = 4, 64
    Lq, Lk = 13 * 12, 126
    q, k, v = make(19, 1, H, Lq, Lk, D, dtype)
    qc, qs = inputs.rope1d(inputs.video_frame_seconds(13, 12), D, bf16=bf)
    kc, ks = inputs.rope1d(inputs.audio_token_seconds(Lk), D, bf16=bf)
    out, _ = AttentionBackend.attention(dev(q, dtype), dev(k, dtype), dev(v, dtype),
                                        q_rotary=Rotary(dev(qc, dtype), dev(qs, dtype)),
                                        k_rotary=Rotary(dev(kc, dtype), dev(ks, dtype)))
    ref, _ = oracle.attention_reference(q, k, v, q_rot=(qc, qs), k_rot=(kc, ks), bf16=bf)
    check(out, ref, dtype, "cross-modal rope")


@pytest.mark.parametrize("name", ["mask_cross_bf16", "mask_cross_fp32", "rope_self_bf16_d128",
                                  "rope_cross_bf16_d64"])
def test_golden_fixtures(golden_dir, name):
    z = np.load(os.path.join(golden_dir, name + ".npz"))
    meta = json.loads(str(z["meta"]))
    dtype = torch.bfloat16 if meta["bf16"] else torch.float32
    s, B, H, Lq, Lk, D = meta["seed"], meta["B"], meta["H"], meta["Lq"], meta["Lk"], meta["D"]
    q = inputs.seeded_tensor(s + 2, (B, H, Lq, D), rmsnorm=meta["rmsnorm"], bf16=meta["bf16"])
    k = inputs.seeded_tensor(s + 3, (B, H, Lk, D), rmsnorm=meta["rmsnorm"], bf16=meta["bf16"])
    v = inputs.seeded_tensor(s + 4, (B, H, Lk, D), bf16=meta["bf16"])
    kw = {}
    if "mask" in z.files:
        kw["key_mask"] = torch.from_numpy(z["mask"]).cuda()
    if "q_cos" in z.files:
        kw["q_rotary"] = Rotary(dev(z["q_cos"], dtype), dev(z["q_sin"], dtype))
    if "k_cos" in z.files:
        kw["k_rotary"] = Rotary(dev(z["k_cos"], dtype), dev(z["k_sin"], dtype))
    out, lse = AttentionBackend.attention(dev(q, dtype), dev(k, dtype), dev(v, dtype), save_lse=True, **kw)
    check(out, z["out"], dtype, name)


@pytest.mark.parametrize("splits", [0, 2, 3, 7, 32])
def test_split_kv_matches_single_pass(splits):
    B, H, Lq, Lk, D = 1, 8, 126, 3120, 64
    q, k, v = make(23, B, H, Lq, Lk, D, torch.bfloat16)
    m = np.ones((B, Lk), np.uint8)
    m[0, 2000:2600] = 0
    qd, kd, vd = dev(q, torch.bfloat16), dev(k, torch.bfloat16), dev(v, torch.bfloat16)
    md = torch.from_numpy(m).cuda()
    out, lse = AttentionBackend.attention(qd, kd, vd, key_mask=md, save_lse=True, num_splits=splits)
    ref, ref_lse = oracle.attn_fwd(q, k, v, mask=m)
    check(out, ref, torch.bfloat16, f"splits={splits}")
    assert np.abs(lse.cpu().numpy() - ref_lse).max() < LSE_ABS
    one, lse1 = AttentionBackend.attention(qd, kd, vd, key_mask=md, save_lse=True, num_splits=1)
    assert (out.float() - one.float()).abs().max().item() <= 2e-2


def _partials_bytes(splits, n_tail, D):
    a256 = lambda x: (x + 255) // 256 * 256
    return a256(splits * n_tail * 256 * D * 4) + a256(splits * n_tail * 256 * 4)


@pytest.mark.parametrize("D,Lq,Lk,extra", [(64, 160, 1024, 12), (128, 256, 2048, 20)])
def test_thin_last_wave_splits_only_the_tail_units(D, Lq, Lk, extra):
    # one 256-row query block per head and sm_count + extra heads: the planner
    # splits the KV range of the `extra` units of the thin last wave only
    sms = device_info()["sm_count"]
    B, H = 1, sms + extra
    q, k, v = make(41, B, H, Lq, Lk, D, torch.bfloat16)
    qd, kd, vd = dev(q, torch.bfloat16), dev(k, torch.bfloat16), dev(v, torch.bfloat16)
    prep = AttentionBackend.prepare(qd, kd, vd, save_lse=True)
    ws = 0 if prep.workspace is None else prep.workspace.numel()
    assert 0 < ws <= _partials_bytes(32, extra, D), ws  # partials of the tail units only
    out, lse = prep.run()
    one, lse1 = AttentionBackend.attention(qd, kd, vd, save_lse=True, num_splits=1)
    assert (out.float() - one.float()).abs().max().item() <= 2e-2
    assert (lse - lse1).abs().max().item() <= LSE_ABS
    # the oracle on the split heads and on a few whole ones
    hs = list(range(H - extra - 4, H))
    ref, ref_lse = oracle.attn_fwd(q[:, hs], k[:, hs], v[:, hs])
    check(out[:, hs], ref, torch.bfloat16, f"D={D} tail heads")
    assert np.abs(lse[:, hs].cpu().numpy() - ref_lse).max() < LSE_ABS


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_transposed_views_need_no_copy(dtype):
    # DiTAttention.swift:346-348: [B, T, H*D] reshaped and transposed to [B, H, T, D]
    B, T, H, D = 2, 200, 4, 64
    base = [torch.from_numpy(inputs.seeded_tensor(31 + i, (B, T, H, D), bf16=dtype == torch.bfloat16)).to(
        "cuda", dtype) for i in range(3)]
    q, k, v = (t.transpose(1, 2) for t in base)
    out_base = torch.empty((B, T, H, D), device="cuda", dtype=dtype)
    out = out_base.transpose(1, 2)
    AttentionBackend.attention(q, k, v, out=out)
    ref, _ = oracle.attn_fwd(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy())
    check(out, ref, dtype, "transposed")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_head_range_computes_only_its_heads(dtype):
    B, H, Lq, Lk, D = 1, 8, 130, 140, 128
    q, k, v = make(37, B, H, Lq, Lk, D, dtype)
    cos, sin = inputs.rope1d(np.arange(max(Lq, Lk), dtype=np.float64), D, bf16=dtype == torch.bfloat16)
    rot = Rotary(dev(cos, dtype), dev(sin, dtype))
    out = torch.full((B, H, Lq, D), 7.0, device="cuda", dtype=dtype)
    lse = torch.full((B, H, Lq), 7.0, device="cuda")
    AttentionBackend.attention(dev(q, dtype), dev(k, dtype), dev(v, dtype), q_rotary=rot, out=out, lse=lse,
                               head_begin=3, head_count=4)
    ref, _ = oracle.attention_reference(q, k, v, q_rot=(cos, sin), bf16=dtype == torch.bfloat16)
    check(out[:, 3:7], ref[:, 3:7], dtype, "head range")
    assert torch.all(out[:, :3] == 7.0) and torch.all(out[:, 7:] == 7.0)
    assert torch.all(lse[:, :3] == 7.0) and torch.all(lse[:, 7:] == 7.0)


def test_config2_full_size_subset_parity_and_properties():
    # BASELINE config 2 at full size: 3120 tokens, 32 heads, D=128, bf16, RMSNorm + 3D RoPE.
    B, H, T, D = 1, 32, 3120, 128
    q, k, v = make(1, B, H, T, T, D, torch.bfloat16)
    cos, sin = inputs.rope3d_grid(13, 12, 20, D)
    rot = Rotary(dev(cos, torch.bfloat16), dev(sin, torch.bfloat16))
    qd, kd, vd = dev(q, torch.bfloat16), dev(k, torch.bfloat16), dev(v, torch.bfloat16)
    out, lse = AttentionBackend.attention(qd, kd, vd, q_rotary=rot, save_lse=True)
    # oracle on two heads (first and last)
    for h in (0, 31):
        ref, ref_lse = oracle.attention_reference(q[:, h:h + 1], k[:, h:h + 1], v[:, h:h + 1], q_rot=(cos, sin),
                                                  bf16=True)
        check(out[:, h:h + 1], ref, torch.bfloat16, f"c2 head {h}")
        assert np.abs(lse[:, h:h + 1].cpu().numpy() - ref_lse).max() < LSE_ABS
    # convexity: every output lies within the per-dim range of v
    o = out.float()
    assert torch.all(o <= vd.float().amax(dim=2, keepdim=True) + 1e-2)
    assert torch.all(o >= vd.float().amin(dim=2, keepdim=True) - 1e-2)
    # permuting keys and values together leaves the output unchanged (rope is applied to
    # the rotated copy first, so permute the un-rotated keys with their table rows)
    perm = torch.randperm(T, generator=torch.Generator().manual_seed(0)).cuda()
    kc = torch.from_numpy(cos).cuda().to(torch.bfloat16)
    ks = torch.from_numpy(sin).cuda().to(torch.bfloat16)
    out_p, _ = AttentionBackend.attention(qd, kd[:, :, perm], vd[:, :, perm], q_rotary=rot,
                                          k_rotary=Rotary(kc[:, :, perm].contiguous(), ks[:, :, perm].contiguous()))
    assert (out_p.float() - o).abs().max().item() <= 2e-2
    # linearity in V: attn(q,k,2v) = 2 attn(q,k,v) exactly in bf16 (power-of-two scaling)
    out_2, _ = AttentionBackend.attention(qd, kd, vd * 2, q_rotary=rot)
    assert torch.equal(out_2.float(), 2 * o)


def test_determinism_bitwise():
    B, H, T, D = 1, 8, 1000, 128
    q, k, v = make(41, B, H, T, T, D, torch.bfloat16)
    qd, kd, vd = dev(q, torch.bfloat16), dev(k, torch.bfloat16), dev(v, torch.bfloat16)
    a, la = AttentionBackend.attention(qd, kd, vd, save_lse=True)
    b, lb = AttentionBackend.attention(qd, kd, vd, save_lse=True)
    assert torch.equal(a, b) and torch.equal(la, lb)


@pytest.mark.parametrize("dtype,D", [(torch.float32, 64), (torch.bfloat16, 128), (torch.bfloat16, 64)])
def test_uniform_attention_is_mean_of_v(dtype, D):
    # q = k = constant: every logit of a row is equal, so O is the mean of the valid V rows
    B, H, L = 1, 2, 300
    q = torch.full((B, H, L, D), 0.25, device="cuda", dtype=dtype)
    v = torch.from_numpy(inputs.seeded_tensor(31, (B, H, L, D), bf16=dtype == torch.bfloat16)).to("cuda", dtype)
    out, _ = AttentionBackend.attention(q, q, v, 1.0 / np.sqrt(D))
    want = v.double().mean(dim=2, keepdim=True).expand(B, H, L, D)
    check(out, want.cpu().numpy(), dtype, "uniform attention")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_one_hot_key_returns_its_value_row(dtype):
    # key 77 aligns with every query and carries a logit ~60 above all others:
    # its softmax weight is 1 to within e^-60, so every output row is V[77]
    B, H, Lq, Lk, D = 1, 2, 130, 200, 64
    g = torch.Generator(device="cpu").manual_seed(3)
    q = torch.zeros((B, H, Lq, D))
    q[..., 0] = 8.0
    k = torch.randn((B, H, Lk, D), generator=g) * 0.01
    k[:, :, 77, 0] = 60.0
    v = torch.randn((B, H, Lk, D), generator=g)
    qd, kd, vd = (t.to("cuda", dtype) for t in (q, k, v))
    out, _ = AttentionBackend.attention(qd, kd, vd, 1.0 / 8.0)
    want = vd[:, :, 77:78, :].double().expand(B, H, Lq, D)
    check(out, want.cpu().numpy(), dtype, "one-hot key")


@pytest.mark.parametrize("dtype,mask", [(torch.bfloat16, False), (torch.bfloat16, True), (torch.float32, True)])
def test_lse_is_log_sum_exp_of_the_logits(dtype, mask):
    # the saved LSE against log(sum_j exp(scale * q.k_j)) over valid keys, computed here in fp64
    B, H, Lq, Lk, D = 2, 2, 260, 390, 64
    q, k, v = make(41, B, H, Lq, Lk, D, dtype)
    qd, kd, vd = dev(q, dtype), dev(k, dtype), dev(v, dtype)
    m = None
    valid = torch.ones((B, Lk), dtype=torch.bool)
    if mask:
        valid[0, 100:] = False
        valid[1, ::3] = False
        m = valid.to("cuda")
    scale = 1.0 / np.sqrt(D)
    _, lse = AttentionBackend.attention(qd, kd, vd, scale, key_mask=m, save_lse=True)
    logits = torch.einsum("bhqd,bhkd->bhqk", qd.double().cpu(), kd.double().cpu()) * scale
    logits = logits.masked_fill(~valid[:, None, None, :], float("-inf"))
    want = torch.logsumexp(logits, dim=-1)
    err = (lse.double().cpu() - want).abs().max().item()
    assert err <= LSE_ABS, f"lse max abs error {err:.3e}"
