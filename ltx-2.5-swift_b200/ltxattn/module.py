"""One DiT attention module on the device: DiTAttention.callAsFunction
(DiTAttention.swift:315-404) with this library between the projections.

    v = linear(kv, to_v)                                   # :341
    q = rmsNorm(linear(x, to_q)), k = rmsNorm(linear(kv, to_k))
    qh, kh = split-RoPE(split(q)), split-RoPE(split(k))    # ltxattn_qk_prep_pair, :358-367
    out = SDPA(qh, kh, split(v), 1/sqrt(D))                # ltxattn_fwd, :369-382
    out = out * 2 sigmoid(linear(x, to_gate_logits))       # fused into ltxattn_fwd's store, :395-399
    return linear(merge(out), to_out.0)                    # merge by view, :401-403

The four projections (and the gate logits) are plain GEMMs and run on the
library GEMM (cuBLAS through torch); the norms, RoPE, attention, gate and merge
run in libltxattn_cuda.  `linear` keeps the reference's two roundings: the
matmul's output in the activation dtype, then the bias added in that dtype
(DiTAttention.swift:178-189).  Weights use the checkpoint's names without the
block prefix: "to_q.weight", "to_q.bias", ..., "q_norm.weight", "k_norm.weight",
and optionally "to_gate_logits.weight" / ".bias".
"""
from __future__ import annotations

import math
from typing import Dict, Optional

import torch

from .backend import AttentionBackend, Failure, Rotary, Variant, qk_prep_pair

NORM_EPS = 1e-6  # DiTAttention.normEpsilon


def linear(x: torch.Tensor, w: Dict[str, torch.Tensor], name: str) -> torch.Tensor:
    """matmul(x, W^T) in the weight dtype, then + bias (DiTAttention.swift:178-189)."""
    weight = w[name + ".weight"]
    y = torch.matmul(x.to(weight.dtype), weight.t())
    b = w.get(name + ".bias")
    if b is not None:
        y = y + b.to(y.dtype)
    return y


class DiTAttentionModule:
    """A DiT attention module's forward on one device (render path).

    ``heads`` is the topology's head count; the head dim comes from ``to_q``
    (DiTAttention.swift:330-336).  ``__call__`` mirrors ``callAsFunction``:
    ``context=None`` is self-attention, ``key_rotary=None`` rotates k with
    ``rotary``, and ``all_perturbed`` returns the gated, merged value stream
    without the q/k work (:349-356).
    """

    def __init__(self, weights: Dict[str, torch.Tensor], heads: int, variant: Variant = Variant.video_self):
        self.w = weights
        self.heads = heads
        self.variant = variant
        q_w = weights["to_q.weight"]
        if q_w.dim() != 2 or q_w.shape[0] % heads:
            raise Failure.shape("to_q.weight", tuple(q_w.shape), f"[k * {heads}, queryDim]")
        self.inner = q_w.shape[0]
        self.head_dim = self.inner // heads

    def __call__(self, x: torch.Tensor, context: Optional[torch.Tensor] = None,
                 rotary: Optional[Rotary] = None, key_rotary: Optional[Rotary] = None,
                 all_perturbed: bool = False) -> torch.Tensor:
        """Runs on torch's current stream (the GEMMs and the library calls alike)."""
        if rotary is not None and not self.variant.takes_rotary:
            raise Failure.rotary_without_position(self.variant)
        w, H, D = self.w, self.heads, self.head_dim
        kv = x if context is None else context
        B, T = x.shape[0], x.shape[1]
        v = linear(kv, w, "to_v")
        vh = v.view(B, kv.shape[1], H, D).permute(0, 2, 1, 3)  # the split view, no copy
        merged = torch.empty((B, T, self.inner), dtype=v.dtype, device=v.device)
        out_view = merged.view(B, T, H, D).permute(0, 2, 1, 3)
        logits = linear(x, w, "to_gate_logits") if "to_gate_logits.weight" in w else None
        if all_perturbed:
            # the value stream itself, gated as the attention output would be
            out = vh
            if logits is not None:
                s = torch.sigmoid(logits.float()).to(v.dtype)
                out = out * (2.0 * s).transpose(1, 2).unsqueeze(-1).to(out.dtype)
            out_view.copy_(out)
        else:
            q = linear(x, w, "to_q")
            k = linear(kv, w, "to_k")
            qh, kh = qk_prep_pair(q, w["q_norm.weight"].to(q.dtype), k, w["k_norm.weight"].to(k.dtype), H,
                                  rotary, key_rotary if key_rotary is not None else rotary, eps=NORM_EPS)
            AttentionBackend.attention(qh, kh, vh, scale=1.0 / math.sqrt(D), out=out_view, gate=logits)
        return linear(merged, w, "to_out.0")
