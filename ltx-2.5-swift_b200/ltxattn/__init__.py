"""ltxattn -- host side of libltxattn_cuda, the B200 fused attention of the
LTX 2.5 DiT (the path of DiTAttention.swift:364-382 in the reference).

    from ltxattn import AttentionBackend, Rotary, scaled_dot_product_attention
"""
from . import _lib
from .backend import (AttentionBackend, Failure, Rotary, Variant, apply_split_rope, device_info,
                      device_status, qk_prep, qk_prep_pair, rotary_tables, scaled_dot_product_attention)
from .module import DiTAttentionModule
from .proj import head_gate, linear

__all__ = ["AttentionBackend", "Failure", "Rotary", "Variant", "scaled_dot_product_attention", "apply_split_rope", "rotary_tables", "qk_prep", "qk_prep_pair",
           "device_info", "device_status", "DiTAttentionModule", "linear", "head_gate", "_lib"]
