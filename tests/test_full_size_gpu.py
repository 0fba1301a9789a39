"""The BASELINE configurations at their stated sizes, through the C ABI, against
the CPU oracle on the same seeded inputs (``ltxattn.workloads``: the inputs the
benchmark times).

* C2 (3120 tokens, 32 heads, D 128, 3D RoPE): every head.
* C3 (3120 queries x 1024 text slots, 94 valid, 32 heads): every head.
* C4a / C4b / C4c (126 audio and 3120 video tokens, 32 heads, D 64, RoPE on
  the shared seconds clock) and the reference-faithful 101-token audio stream:
  every head.
* C5 (29,760 tokens, D 128), one 4-head block of the 8-GPU shard: the forward
  of head 0 over all rows and of head 3 on a row sample; the backward of
  head 0 with dQ on a row sample and dK / dV on a key sample (the oracle
  streams over rows; it holds no 29,760 x 29,760 matrix).

Tolerances: bf16 max abs <= 2e-2 and rel-L2 <= 1e-2
against the fp64-accumulated oracle; gradients as in test_bwd_gpu.py.
"""
import numpy as np
import pytest
import torch

import oracle
from ltxattn import AttentionBackend, Rotary, device_status, workloads

pytestmark = pytest.mark.gpu

BF16_MAX_ABS = 2e-2
BF16_REL_L2 = 1e-2
LSE_ABS = 2e-3


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda", torch.bfloat16)


def check(got, ref, what):
    g = got.float().cpu().numpy() if isinstance(got, torch.Tensor) else got
    err = np.abs(g.astype(np.float64) - ref.astype(np.float64))
    rel = float(np.linalg.norm(err) / max(np.linalg.norm(ref), 1e-30))
    assert err.max() <= BF16_MAX_ABS and rel <= BF16_REL_L2, f"{what}: max abs {err.max():.3e} rel-L2 {rel:.3e}"


def check_grad(got, ref, what):
    g = got.float().cpu().numpy().astype(np.float64) if isinstance(got, torch.Tensor) else got.astype(np.float64)
    r = ref.astype(np.float64)
    err = np.abs(g - r)
    scale = max(1.0, float(np.abs(r).max()))
    rel = float(np.linalg.norm(err) / max(np.linalg.norm(r), 1e-3 * np.sqrt(r.size)))
    assert err.max() <= 2e-2 * scale and rel <= 1e-2, f"{what}: max abs {err.max():.3e} rel-L2 {rel:.3e}"


@pytest.fixture(autouse=True)
def no_kernel_timeouts():
    yield
    assert device_status(clear=True) == 0, "a kernel wait timed out"


def run_forward(w, q, k, v, tabs, mask):
    qr = kr = None
    if tabs is not None:
        qr = Rotary(dev(tabs[0][0]), dev(tabs[0][1]))
        if tabs[1] is not None:
            kr = Rotary(dev(tabs[1][0]), dev(tabs[1][1]))
    md = torch.from_numpy(mask).cuda() if mask is not None else None
    out, lse = AttentionBackend.attention(dev(q), dev(k), dev(v), key_mask=md, q_rotary=qr, k_rotary=kr,
                                          save_lse=True)
    return out, lse


def oracle_forward(q, k, v, tabs, mask):
    q_rot = k_rot = None
    if tabs is not None:
        q_rot, k_rot = tabs
    return oracle.attention_reference(q, k, v, mask=mask, q_rot=q_rot, k_rot=k_rot, bf16=True)


@pytest.mark.parametrize("name", ["c2", "c3", "c4a", "c4b", "c4c", "a101"])
def test_config_at_full_size_every_head(name):
    w = workloads.WORKLOADS[name]
    q, k, v, tabs, mask = workloads.host_inputs(w)
    out, lse = run_forward(w, q, k, v, tabs, mask)
    torch.cuda.synchronize()
    ref, ref_lse = oracle_forward(q, k, v, tabs, mask)
    check(out, ref, f"{name} all {w.H} heads")
    assert np.abs(lse.cpu().numpy() - ref_lse).max() < LSE_ABS
    # each head on its own, so one bad head cannot hide in the aggregate
    got = out.float().cpu().numpy()
    for h in range(w.H):
        check(got[:, h], ref[:, h], f"{name} head {h}")


def test_config3_masked_keys_carry_no_weight():
    # the 930 padded slots of config 3 cannot influence the output: rewriting
    # their keys and values leaves every bit unchanged
    w = workloads.WORKLOADS["c3"]
    q, k, v, _, mask = workloads.host_inputs(w, heads=(0, 8))
    md = torch.from_numpy(mask).cuda()
    a, _ = AttentionBackend.attention(dev(q), dev(k), dev(v), key_mask=md)
    k2, v2 = k.copy(), v.copy()
    k2[:, :, w.mask_valid:] = 7.0
    v2[:, :, w.mask_valid:] = -3.0
    b, _ = AttentionBackend.attention(dev(q), dev(k2), dev(v2), key_mask=md)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def _c5_rows(T):
    mid = T // 2 - 128
    return np.concatenate([np.arange(0, 128), np.arange(mid, mid + 256), np.arange(T - 128, T)])


def _c5_keys(T):
    mid = T // 2 - 32
    return np.concatenate([np.arange(0, 128), np.arange(mid, mid + 64), np.arange(T - 64, T)])


def test_config5_forward_and_backward_on_one_shard():
    # 29,760 tokens, heads 0..3 of the 32 (one rank's block at 8 GPUs), no RoPE, plain N(0,1)
    w = workloads.WORKLOADS["c5"]
    hc = 4
    q, k, v, _, _ = workloads.host_inputs(w, heads=(0, hc))
    do = workloads.host_dout(w, heads=(0, hc))
    qd, kd, vd, dod = dev(q), dev(k), dev(v), dev(do)
    out, lse = AttentionBackend.attention(qd, kd, vd, save_lse=True)
    dq, dk, dv = AttentionBackend.attention_backward(qd, kd, vd, out, dod, lse)
    torch.cuda.synchronize()
    T = w.Lq
    rows = _c5_rows(T)
    keys = _c5_keys(T)
    rows_d = torch.as_tensor(rows, device="cuda")
    keys_d = torch.as_tensor(keys, device="cuda")

    # forward, head 0: every row
    ref0, ref_lse0 = oracle.attn_fwd(q[:, :1], k[:, :1], v[:, :1])
    check(out[:, :1], ref0, "c5 head 0 forward")
    assert np.abs(lse[:, :1].cpu().numpy() - ref_lse0).max() < LSE_ABS
    # forward, head 3: the row sample
    ref3, ref_lse3 = oracle.attn_fwd(q[:, 3:4, rows], k[:, 3:4], v[:, 3:4])
    check(out[:, 3:4][:, :, rows_d], ref3, "c5 head 3 forward (rows)")
    assert np.abs(lse[:, 3:4][:, :, rows_d].cpu().numpy() - ref_lse3).max() < LSE_ABS

    # backward, head 0: dQ of the sampled rows (each row's gradient needs only that row)
    rdq, _, _ = oracle.attn_bwd(q[:, :1, rows], k[:, :1], v[:, :1], do[:, :1, rows])
    check_grad(dq[:, :1][:, :, rows_d], rdq, "c5 dq (rows)")
    # dK / dV of the sampled keys, with the oracle's own lse and delta over all rows
    delta = np.sum(ref0[0, 0].astype(np.float64) * do[0, 0], axis=-1)
    rdk, rdv = oracle.attn_bwd_keys(q[0, 0], k[0, 0], v[0, 0], do[0, 0], ref_lse0[0, 0], delta, keys)
    check_grad(dk[0, 0][keys_d], rdk, "c5 dk (keys)")
    check_grad(dv[0, 0][keys_d], rdv, "c5 dv (keys)")
