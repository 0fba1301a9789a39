"""Generate the golden fixtures in this folder.

The reference (Swift + MLX on Metal) cannot run on this machine, so these
vectors come from an implementation that is independent of both the CUDA
kernels and the C oracle: torch in float64 on the CPU, written directly from
the reference's explicit attention arm and its mask convention:

* ``Sources/LTXModules/DiTAttention.swift:377-381``
  logits = q.k^T * scale; softmax(-1); @ v
* ``Sources/LTXModules/DiTAttention.swift:226-234``  split RoPE, evaluated on
  bf16 tensors when the case is bf16 (torch's bf16 CPU ops round each result,
  as MLX's do)
* ``Sources/LTXModules/GemmaTextEncoder.swift:304-323``  additive mask of
  -FLT_MAX for masked keys; rows with no allowed key are un-masked
* gradients by torch autograd in float64 (the reference's backward is MLX
  autodiff, ``LoRATrainingStep.swift:283-304``)

Inputs are regenerated from seeds by ``ltxattn.inputs`` (the package's
counter-based splitmix64 + Box-Muller stream); each fixture stores the seeds,
a sha256 of the input bytes (so a drifting generator is caught) and the
outputs.  Run:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "ltx-2.5-swift_b200"))
from ltxattn import inputs  # noqa: E402

FLT_MAX = float(np.finfo(np.float32).max)


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a, dtype=np.float32).tobytes())
    return h.hexdigest()


def torch_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    cos, sin = cos.to(x.dtype), sin.to(x.dtype)
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


def torch_sdpa(q, k, v, mask, scale):
    logits = torch.matmul(q, k.transpose(-1, -2)) * scale
    if mask is not None:
        allowed = torch.as_tensor(mask != 0)[:, None, None, :].expand(logits.shape)
        any_allowed = allowed.any(dim=-1, keepdim=True)
        allowed = allowed | ~any_allowed
        logits = logits + torch.where(allowed, 0.0, -FLT_MAX).to(logits.dtype)
    return torch.matmul(torch.softmax(logits, dim=-1), v), torch.logsumexp(logits, dim=-1)


def make_case(name, B, H, Lq, Lk, D, *, seed, bf16, rmsnorm=False, mask=None,
              q_tab=None, k_tab=None, grad=False):
    q = inputs.seeded_tensor(seed + 2, (B, H, Lq, D), rmsnorm=rmsnorm, bf16=bf16)
    k = inputs.seeded_tensor(seed + 3, (B, H, Lk, D), rmsnorm=rmsnorm, bf16=bf16)
    v = inputs.seeded_tensor(seed + 4, (B, H, Lk, D), bf16=bf16)
    dout = inputs.seeded_tensor(seed + 5, (B, H, Lq, D), bf16=bf16) if grad else None
    scale = 1.0 / np.sqrt(D)
    tq = torch.from_numpy(q).double().requires_grad_(grad)
    tk = torch.from_numpy(k).double().requires_grad_(grad)
    tv = torch.from_numpy(v).double().requires_grad_(grad)
    qr, kr = tq, tk
    rec = {}
    if q_tab is not None:
        kt = k_tab if k_tab is not None else q_tab
        if bf16:
            # bf16 arithmetic as the reference does it; the rotated tensors are
            # the SDPA inputs, carried on in float64 for the attention itself.
            qr_b = torch_rope(torch.from_numpy(q).bfloat16(), torch.from_numpy(q_tab[0]),
                              torch.from_numpy(q_tab[1]))
            kr_b = torch_rope(torch.from_numpy(k).bfloat16(), torch.from_numpy(kt[0]),
                              torch.from_numpy(kt[1]))
            rec["q_rotated"] = qr_b.float().numpy()
            rec["k_rotated"] = kr_b.float().numpy()
            if grad:
                # straight-through the bf16 roundings, as autodiff does
                qr = torch_rope(tq, torch.from_numpy(q_tab[0]).double(), torch.from_numpy(q_tab[1]).double())
                kr = torch_rope(tk, torch.from_numpy(kt[0]).double(), torch.from_numpy(kt[1]).double())
                qr = qr + (torch.from_numpy(rec["q_rotated"]).double() - qr).detach()
                kr = kr + (torch.from_numpy(rec["k_rotated"]).double() - kr).detach()
            else:
                qr = qr_b.double()
                kr = kr_b.double()
        else:
            qr = torch_rope(tq, torch.from_numpy(q_tab[0]).double(), torch.from_numpy(q_tab[1]).double())
            kr = torch_rope(tk, torch.from_numpy(kt[0]).double(), torch.from_numpy(kt[1]).double())
            rec["q_rotated"] = qr.detach().float().numpy()
            rec["k_rotated"] = kr.detach().float().numpy()
    out, lse = torch_sdpa(qr, kr, tv, mask, scale)
    rec["out"] = out.detach().float().numpy()
    rec["lse"] = lse.detach().float().numpy()
    if grad:
        out.backward(torch.from_numpy(dout).double())
        rec["dq"] = tq.grad.float().numpy()
        rec["dk"] = tk.grad.float().numpy()
        rec["dv"] = tv.grad.float().numpy()
    meta = dict(name=name, B=B, H=H, Lq=Lq, Lk=Lk, D=D, seed=seed, bf16=bf16,
                rmsnorm=rmsnorm, grad=grad, input_sha256=sha(q, k, v, *( [dout] if grad else [])))
    arrays = {kk: vv for kk, vv in rec.items()}
    if mask is not None:
        arrays["mask"] = mask.astype(np.uint8)
    if q_tab is not None:
        arrays["q_cos"], arrays["q_sin"] = q_tab
        if k_tab is not None:
            arrays["k_cos"], arrays["k_sin"] = k_tab
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), meta=json.dumps(meta), **arrays)
    return meta


def main():
    torch.manual_seed(0)
    metas = []
    # BASELINE config 1 itself: fp32, B1 H4 256x256 D64, no mask, no RoPE.
    metas.append(make_case("c1_fp32_256", 1, 4, 256, 256, 64, seed=1000, bf16=False))
    # ragged cross attention with a key-padding mask; batch 1 is fully masked
    # (the un-mask rule), batch 0 keeps 19 of 53 keys.
    m = np.zeros((2, 53), np.uint8)
    m[0, :19] = 1
    metas.append(make_case("mask_cross_bf16", 2, 3, 37, 53, 64, seed=2000, bf16=True,
                           rmsnorm=True, mask=m))
    metas.append(make_case("mask_cross_fp32", 2, 3, 37, 53, 64, seed=2100, bf16=False, mask=m))
    # self attention, D=128, per-head distinct tables from the reference's own builder
    pos = inputs.video_positions(3, 3, 5)
    tab = inputs.reference_rotary(pos, inner=4 * 128, max_pos=[20, 2048, 2048], heads=4)
    metas.append(make_case("rope_self_bf16_d128", 1, 4, 45, 45, 128, seed=3000, bf16=True,
                           rmsnorm=True, q_tab=tab))
    # cross-modal: separate query / key tables on a shared seconds clock
    qt = inputs.rope1d(inputs.video_frame_seconds(3, 10), 64)
    kt = inputs.rope1d(inputs.audio_token_seconds(41), 64)
    metas.append(make_case("rope_cross_bf16_d64", 1, 2, 30, 41, 64, seed=4000, bf16=True,
                           rmsnorm=True, q_tab=qt, k_tab=kt))
    # gradients: masked, and with RoPE
    m2 = np.zeros((1, 47), np.uint8)
    m2[0, :31] = 1
    metas.append(make_case("grad_mask_fp32", 1, 2, 33, 47, 64, seed=5000, bf16=False, mask=m2,
                           grad=True))
    gt = inputs.rope1d(np.arange(40, dtype=np.float64), 64, bf16=False)
    metas.append(make_case("grad_rope_fp32", 1, 2, 40, 40, 64, seed=6000, bf16=False,
                           q_tab=gt, grad=True))
    with open(os.path.join(HERE, "manifest.json"), "w") as f:
        json.dump(metas, f, indent=1)
    print(f"wrote {len(metas)} fixtures")


if __name__ == "__main__":
    main()
