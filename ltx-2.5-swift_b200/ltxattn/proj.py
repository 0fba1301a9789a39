"""The attention module's projections through libltxattn_cuda's tcgen05 GEMMs.

* ``linear(x, weight, bias)`` is ``DiTAttention.linear`` (DiTAttention.swift:178-188,
  without the LoRA overlay): ``T(T(x W^T) + b)`` through ``ltxattn_linear``.
* ``head_gate(x, logits, out)`` is the per-head gate and merge of the STG
  passthrough (:349-356, 395-403) through ``ltxattn_head_gate``.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib
from .backend import Failure, _stream_ptr, _view


def _need_bf16(name: str, t: torch.Tensor):
    if not t.is_cuda:
        raise Failure("arg", f"{name} must be a CUDA tensor", _lib.ERR_ARG)
    if t.dtype != torch.bfloat16:
        raise Failure("dtype", f"{name} must be bfloat16", _lib.ERR_DTYPE)


def linear(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
           out: Optional[torch.Tensor] = None, stream=None, split_k: bool = True) -> torch.Tensor:
    """x [..., k] (rows with one stride, unit stride along k), weight [n, k] -> [..., n].

    A narrow output (few column tiles) gets the workspace ltxattn_linear asks
    for and splits K across CTAs, unless ``split_k`` is False."""
    _need_bf16("x", x)
    _need_bf16("weight", weight)
    k = x.shape[-1]
    n = weight.shape[0]
    if weight.dim() != 2 or weight.shape[1] != k or weight.stride(1) != 1:
        raise Failure.shape("weight", weight.shape, f"[n, {k}] with unit stride along k")
    x2 = x.reshape(-1, k)  # a view when the leading dims collapse into one row stride
    if x2.stride(1) != 1:
        raise Failure("align", "x must have unit stride along its last dim", _lib.ERR_ALIGN)
    m = x2.shape[0]
    if out is None:
        out = torch.empty(x.shape[:-1] + (n,), dtype=x.dtype, device=x.device)
    o2 = out.view(-1, n)
    a = _lib.LinearArgs()
    a.dtype, a.m, a.n, a.k = _lib.BF16, m, n, k
    a.x, a.x_stride = x2.data_ptr(), x2.stride(0) if m > 1 else k
    a.weight, a.weight_stride = weight.data_ptr(), weight.stride(0)
    if bias is not None:
        _need_bf16("bias", bias)
        if bias.numel() != n or not bias.is_contiguous():
            raise Failure.shape("bias", bias.shape, f"[{n}] contiguous")
        a.bias = bias.data_ptr()
    a.out, a.out_stride = o2.data_ptr(), o2.stride(0) if m > 1 else n
    L = _lib.load()
    ws_bytes = int(L.ltxattn_linear_workspace(ctypes.byref(a)))
    ws = None
    if ws_bytes and split_k:
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)  # a narrow output splits K
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws_bytes
    rc = L.ltxattn_linear(ctypes.byref(a), ctypes.c_void_p(_stream_ptr(stream)))
    if rc != _lib.OK:
        raise Failure.from_status(rc)
    return out


def head_gate(x: torch.Tensor, logits: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
              stream=None) -> torch.Tensor:
    """x [B, H, T, D] -> T(T(x) * 2 T(sigmoid(logits))) per head (logits [B, T, H]; None:
    a copy), into ``out`` (may view the merged [B, T, H * D] buffer)."""
    if x.dim() != 4:
        raise Failure.shape("x", x.shape, "[B, heads, tokens, headDim]")
    B, H, T, D = x.shape
    if out is None:
        out = torch.empty_like(x)
    a = _lib.HeadGateArgs()
    a.dtype = _lib.BF16 if x.dtype == torch.bfloat16 else _lib.F32
    a.batch, a.heads, a.tokens, a.head_dim = B, H, T, D
    a.x, a.out = _view("x", x, (B, H, T, D)), _view("out", out, (B, H, T, D))
    if logits is not None:
        if tuple(logits.shape) != (B, T, H) or logits.dtype != x.dtype:
            raise Failure.shape("logits", logits.shape, f"[{B}, {T}, {H}] {x.dtype}")
        a.gate = logits.data_ptr()
        a.gate_stride_b, a.gate_stride_t, a.gate_stride_h = logits.stride(0), logits.stride(1), logits.stride(2)
    rc = _lib.load().ltxattn_head_gate(ctypes.byref(a), ctypes.c_void_p(_stream_ptr(stream)))
    if rc != _lib.OK:
        raise Failure.from_status(rc)
    return out
