"""One DiT attention module on the device: DiTAttention.callAsFunction
(DiTAttention.swift:315-404), every step in libltxattn_cuda.

    v = linear(kv, to_v)                                   # ltxattn_linear, :341
    q, k = linear(x, to_q), linear(kv, to_k)               # ltxattn_linear, :342
    qh, kh = split-RoPE(split(rmsNorm(q, k)))              # ltxattn_qk_prep_pair, :358-367
    out = SDPA(qh, kh, split(v), 1/sqrt(D))                # ltxattn_fwd, :369-382
    out = out * 2 sigmoid(linear(x, to_gate_logits))       # fused into ltxattn_fwd's store, :395-399
    return linear(merge(out), to_out.0)                    # merge by view, :401-403

The projections run on the library's tcgen05 GEMMs (``gemm="ltxattn"``, the
default) or, for comparison, on the library GEMM of torch (``gemm="torch"``:
cuBLAS).  Either way ltxattn_qk_prep_pair applies the norms, the head split
and RoPE to q and k in one launch.  `linear` keeps the
reference's two roundings either way: the matmul's output in the activation
dtype, then the bias added in that dtype (DiTAttention.swift:178-189).  The STG
passthrough (all_perturbed, :349-356) gates and merges the value stream with
ltxattn_head_gate.  Weights use the checkpoint's names without the block
prefix: "to_q.weight", "to_q.bias", ..., "q_norm.weight", "k_norm.weight",
and optionally "to_gate_logits.weight" / ".bias".
"""
from __future__ import annotations

import math
from typing import Dict, Optional

import torch

from . import proj
from .backend import AttentionBackend, Failure, Rotary, Variant, qk_prep_pair

NORM_EPS = 1e-6  # DiTAttention.normEpsilon


def linear(x: torch.Tensor, w: Dict[str, torch.Tensor], name: str, gemm: str = "ltxattn") -> torch.Tensor:
    """matmul(x, W^T) in the weight dtype, then + bias (DiTAttention.swift:178-189)."""
    weight = w[name + ".weight"]
    b = w.get(name + ".bias")
    if gemm == "ltxattn":
        return proj.linear(x.to(weight.dtype), weight, b.to(weight.dtype) if b is not None else None)
    y = torch.matmul(x.to(weight.dtype), weight.t())
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

    def __init__(self, weights: Dict[str, torch.Tensor], heads: int, variant: Variant = Variant.video_self,
                 gemm: str = "ltxattn"):
        if gemm not in ("ltxattn", "torch"):
            raise Failure("arg", f"gemm must be 'ltxattn' or 'torch', not {gemm!r}")
        self.w = weights
        self.heads = heads
        self.variant = variant
        self.gemm = gemm
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
        w, H, D, g = self.w, self.heads, self.head_dim, self.gemm
        kv = x if context is None else context
        B, T = x.shape[0], x.shape[1]
        v = linear(kv, w, "to_v", g)
        vh = v.view(B, kv.shape[1], H, D).permute(0, 2, 1, 3)  # the split view, no copy
        merged = torch.empty((B, T, self.inner), dtype=v.dtype, device=v.device)
        out_view = merged.view(B, T, H, D).permute(0, 2, 1, 3)
        logits = linear(x, w, "to_gate_logits", g) if "to_gate_logits.weight" in w else None
        if all_perturbed:
            # the value stream itself, gated as the attention output would be, into the merged buffer
            proj.head_gate(vh, logits, out=out_view)
        else:
            k_rot = key_rotary if key_rotary is not None else rotary
            q = linear(x, w, "to_q", g)
            k = linear(kv, w, "to_k", g)
            qh, kh = qk_prep_pair(q, w["q_norm.weight"].to(q.dtype), k, w["k_norm.weight"].to(k.dtype), H,
                                  rotary, k_rot, eps=NORM_EPS)
            AttentionBackend.attention(qh, kh, vh, scale=1.0 / math.sqrt(D), out=out_view, gate=logits)
        return linear(merged, w, "to_out.0", g)
