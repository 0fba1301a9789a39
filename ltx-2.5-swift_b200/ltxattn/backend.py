"""Host-side mirror of the reference's attention seam, over the C ABI.

The reference's seam is ``Sources/LTXAttention`` (``AttentionBackend.swift:13-15``,
a placeholder) and the call it stands in for is the SDPA switch of
``Sources/LTXModules/DiTAttention.swift:369-382``:

    MLXFast.scaledDotProductAttention(queries:keys:values:scale:mask:)

preceded by ``applySplitRoPE`` (``:364-367``).  This module keeps those names
and meanings:

* ``scaled_dot_product_attention(queries, keys, values, scale, mask=None)`` is
  the MLXFast call (``mask`` here is a boolean key-padding mask ``[B, Lk]``).
* ``AttentionBackend.attention(q, k, v, scale, key_mask, q_rotary, k_rotary,
  save_lse)`` is the fused RoPE + SDPA entry the Swift shim exposes, with
  ``k_rotary=None`` meaning "use q_rotary for k" (``keyRotary ?? rotary``).
* ``AttentionBackend.attention_backward(...)`` is the VJP the LoRA trainer
  needs (``LoRATrainingStep.swift:283-304``).
* ``Rotary`` is ``DiTAttention.Rotary`` (``:98-105``); ``Variant`` and
  ``Failure`` mirror ``DiTAttention.Variant`` (``:69-90``) and
  ``DiTAttention.Failure`` (``:107-122``).

Tensors are torch CUDA tensors (PyTorch provides device memory and streams);
``[B, H, T, D]`` views may be strided, as the reference's transposed ``split``
views are.  Every call goes through ``libltxattn_cuda``; there is no other
implementation behind it.
"""
from __future__ import annotations

import ctypes
import enum
import math
from dataclasses import dataclass
from typing import Optional, Tuple

import torch

from . import _lib


class Failure(Exception):
    """DiTAttention.Failure plus the library's status codes.

    ``kind`` is one of ``missing``, ``shape``, ``rotaryWithoutPosition`` (the
    reference's cases) or the C ABI's status names (``dtype``, ``align``,
    ``unsupported``, ``cuda``, ``nccl``, ``timeout``, ``workspace``, ``arg``).
    """

    def __init__(self, kind: str, message: str, status: int = -1):
        super().__init__(message)
        self.kind = kind
        self.status = status

    @classmethod
    def shape(cls, name: str, got, expected: str) -> "Failure":
        # DiTAttention.swift:115-116: "\(name) is \(got), expected \(expected)"
        return cls("shape", f"{name} is {list(got)}, expected {expected}", _lib.ERR_SHAPE)

    @classmethod
    def rotary_without_position(cls, variant: "Variant") -> "Failure":
        return cls("rotaryWithoutPosition",
                   f"{variant.value} takes no rotary embedding; supplying one would rotate a "
                   "stream that has no latent position")

    @classmethod
    def from_status(cls, status: int) -> "Failure":
        return cls(_lib.STATUS_NAMES.get(status, str(status)), _lib.last_error(), status)


class Variant(enum.Enum):
    """The six attention modules of a DiT block (DiTAttention.swift:69-90)."""

    video_self = "attn1"
    video_cross = "attn2"
    audio_self = "audio_attn1"
    audio_cross = "audio_attn2"
    audio_to_video = "audio_to_video_attn"
    video_to_audio = "video_to_audio_attn"

    @property
    def takes_rotary(self) -> bool:
        return self not in (Variant.video_cross, Variant.audio_cross)


@dataclass
class Rotary:
    """(cos, sin), each [B, heads, tokens, D/2] (broadcast dims may be size 1)."""

    cos: torch.Tensor
    sin: torch.Tensor


def _check_cuda(name: str, t: torch.Tensor):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise Failure("arg", f"{name} must be a CUDA tensor", _lib.ERR_ARG)


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return _lib.BF16
    if t.dtype == torch.float32:
        return _lib.F32
    raise Failure("dtype", f"dtype {t.dtype} is neither bfloat16 nor float32", _lib.ERR_DTYPE)


def _view(name: str, t: torch.Tensor, shape) -> _lib.Tensor:
    if t.dim() != 4 or tuple(t.shape) != tuple(shape):
        raise Failure.shape(name, t.shape, str(list(shape)))
    if t.stride(3) != 1:
        raise Failure("align", f"{name} must have a unit stride in its last dim", _lib.ERR_ALIGN)
    return _lib.Tensor(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2))


def _rotary(name: str, r: Optional[Rotary], B: int, H: int, T: int, D: int, dtype) -> _lib.Rotary:
    if r is None:
        return _lib.Rotary()
    for part, t in (("cos", r.cos), ("sin", r.sin)):
        _check_cuda(f"{name}.{part}", t)
        if t.dtype != dtype:
            raise Failure("dtype", f"{name}.{part} is {t.dtype}; the reference narrows tables to the "
                          f"activation dtype {dtype}", _lib.ERR_DTYPE)
        if t.dim() != 4 or t.shape[-1] != D // 2 or t.shape[0] not in (1, B) or t.shape[1] not in (1, H):
            raise Failure.shape(f"{name}.{part}", t.shape, f"[1|{B}, 1|{H}, >={T}, {D // 2}]")
        if t.stride(3) != 1:
            raise Failure("align", f"{name}.{part} must have a unit stride in its last dim", _lib.ERR_ALIGN)
    if r.cos.shape != r.sin.shape or r.cos.stride() != r.sin.stride():
        raise Failure.shape(f"{name}.sin", r.sin.shape, f"the layout of {name}.cos {list(r.cos.shape)}")
    c = r.cos
    sb = 0 if c.shape[0] == 1 else c.stride(0)
    sh = 0 if c.shape[1] == 1 else c.stride(1)
    return _lib.Rotary(c.data_ptr(), r.sin.data_ptr(), sb, sh, c.stride(2), c.shape[2])


def _stream_ptr(stream) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


class AttentionBackend:
    """The attention seam, backed by libltxattn_cuda."""

    @staticmethod
    def workspace_bytes(args: _lib.FwdArgs) -> int:
        return int(_lib.load().ltxattn_fwd_workspace(ctypes.byref(args)))

    @staticmethod
    def make_fwd_args(q, k, v, scale, key_mask=None, q_rotary=None, k_rotary=None, lse=None,
                      out=None, head_begin=0, head_count=0, num_splits=0, causal=False,
                      window=0, gate=None) -> Tuple[_lib.FwdArgs, torch.Tensor]:
        for name, t in (("q", q), ("k", k), ("v", v)):
            _check_cuda(name, t)
        if q.dim() != 4:
            raise Failure.shape("q", q.shape, "[B, heads, tokens, headDim]")
        B, H, Lq, D = q.shape
        # k / v may carry fewer heads than q (grouped KV heads, the Gemma encoder's GQA)
        if k.dim() != 4 or k.shape[0] != B or k.shape[1] < 1 or H % k.shape[1] or k.shape[3] != D:
            raise Failure.shape("k", k.shape, f"[{B}, {H} or a divisor of it, kvTokens, {D}]")
        Hk = k.shape[1]
        Lk = k.shape[2]
        dt = _dtype_code(q)
        if k.dtype != q.dtype or v.dtype != q.dtype:
            raise Failure("dtype", "q, k and v must share one dtype", _lib.ERR_DTYPE)
        if out is None:
            out = torch.empty((B, H, Lq, D), dtype=q.dtype, device=q.device)
        a = _lib.FwdArgs()
        a.dtype = dt
        a.batch, a.heads, a.q_len, a.kv_len, a.head_dim = B, H, Lq, Lk, D
        a.head_begin, a.head_count = head_begin, head_count
        a.q = _view("q", q, (B, H, Lq, D))
        a.k = _view("k", k, (B, Hk, Lk, D))
        a.v = _view("v", v, (B, Hk, Lk, D))
        a.out = _view("out", out, (B, H, Lq, D))
        a.scale = float(scale)
        if key_mask is not None:
            _check_cuda("key_mask", key_mask)
            if key_mask.dtype not in (torch.bool, torch.uint8) or tuple(key_mask.shape) != (B, Lk):
                raise Failure.shape("key_mask", key_mask.shape, f"[{B}, {Lk}] bool")
            if key_mask.stride(1) != 1:
                raise Failure("align", "key_mask must be contiguous along keys", _lib.ERR_ALIGN)
            a.key_mask = key_mask.data_ptr()
            a.key_mask_stride_b = key_mask.stride(0)
        a.q_rotary = _rotary("q_rotary", q_rotary, B, H, Lq, D, q.dtype)
        a.k_rotary = _rotary("k_rotary", k_rotary, B, H, Lk, D, q.dtype)
        if lse is not None:
            _check_cuda("lse", lse)
            if lse.dtype != torch.float32 or tuple(lse.shape) != (B, H, Lq) or lse.stride(2) != 1:
                raise Failure.shape("lse", lse.shape, f"[{B}, {H}, {Lq}] float32, contiguous rows")
            a.lse = lse.data_ptr()
            a.lse_stride_b, a.lse_stride_h = lse.stride(0), lse.stride(1)
        a.num_splits = num_splits
        a.causal, a.window, a.kv_heads = int(bool(causal)), int(window), Hk
        if gate is not None:
            # to_gate_logits output [B, tokens, heads] (DiTAttention.swift:395-399), any strides
            _check_cuda("gate", gate)
            if tuple(gate.shape) != (B, Lq, H) or gate.dtype != q.dtype:
                raise Failure.shape("gate", gate.shape, f"[{B}, {Lq}, {H}] {q.dtype}")
            a.gate = gate.data_ptr()
            a.gate_stride_b, a.gate_stride_t, a.gate_stride_h = gate.stride(0), gate.stride(1), gate.stride(2)
        return a, out

    @staticmethod
    def prepare(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: Optional[float] = None,
                key_mask: Optional[torch.Tensor] = None, q_rotary: Optional[Rotary] = None,
                k_rotary: Optional[Rotary] = None, save_lse: bool = False, head_begin: int = 0,
                head_count: int = 0, num_splits: int = 0, out: Optional[torch.Tensor] = None,
                lse: Optional[torch.Tensor] = None, gate: Optional[torch.Tensor] = None) -> "PreparedAttention":
        """Validate and marshal once; ``run()`` then issues just ``ltxattn_fwd``.

        For repeated calls on the same buffers (a render loop, a benchmark): the
        argument block and the workspace are built here and reused by every run.
        """
        if scale is None:
            scale = 1.0 / math.sqrt(q.shape[-1])
        if save_lse and lse is None:
            lse = torch.empty(q.shape[:3], dtype=torch.float32, device=q.device)
        a, out = AttentionBackend.make_fwd_args(q, k, v, scale, key_mask, q_rotary, k_rotary, lse, out,
                                                head_begin, head_count, num_splits, gate=gate)
        return PreparedAttention(a, out, lse, (q, k, v, key_mask, q_rotary, k_rotary, gate))

    @staticmethod
    def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: Optional[float] = None,
                  key_mask: Optional[torch.Tensor] = None, q_rotary: Optional[Rotary] = None,
                  k_rotary: Optional[Rotary] = None, save_lse: bool = False,
                  variant: Optional[Variant] = None, head_begin: int = 0, head_count: int = 0,
                  num_splits: int = 0, out: Optional[torch.Tensor] = None,
                  lse: Optional[torch.Tensor] = None, stream=None, causal: bool = False, window: int = 0,
                  gate: Optional[torch.Tensor] = None):
        """Fused split-RoPE + SDPA.  Returns ``(out, lse)``; lse is None unless requested.

        ``causal`` / ``window`` / grouped KV heads (``k`` with fewer heads than ``q``)
        give the Gemma text encoder's self-attention (GemmaTextEncoder.swift:218-233,
        292-323); the DiT's attention uses none of them.  ``gate`` ([B, tokens, heads]
        ``to_gate_logits`` output) fuses the per-head gate out * 2*sigmoid(logit)
        (DiTAttention.swift:395-399) into the store; ``out`` may be the merged
        [B, tokens, heads * headDim] buffer seen as [B, heads, tokens, headDim].
        """
        if variant is not None and q_rotary is not None and not variant.takes_rotary:
            raise Failure.rotary_without_position(variant)
        if scale is None:
            scale = 1.0 / math.sqrt(q.shape[-1])  # DiTAttention.swift:372
        if save_lse and lse is None:
            lse = torch.empty(q.shape[:3], dtype=torch.float32, device=q.device)
        a, out = AttentionBackend.make_fwd_args(q, k, v, scale, key_mask, q_rotary, k_rotary, lse, out,
                                                head_begin, head_count, num_splits, causal, window, gate)
        L = _lib.load()
        ws_bytes = int(L.ltxattn_fwd_workspace(ctypes.byref(a)))
        ws = None
        if ws_bytes > 0:
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
            a.workspace, a.workspace_bytes = ws.data_ptr(), ws_bytes
        rc = L.ltxattn_fwd(ctypes.byref(a), ctypes.c_void_p(_stream_ptr(stream)))
        if rc != _lib.OK:
            raise Failure.from_status(rc)
        return out, lse

    @staticmethod
    def attention_backward(q, k, v, out, dout, lse, scale: Optional[float] = None,
                           key_mask=None, q_rotary: Optional[Rotary] = None,
                           k_rotary: Optional[Rotary] = None, head_begin: int = 0, head_count: int = 0,
                           dq=None, dk=None, dv=None, stream=None):
        """Gradients (dq, dk, dv) of sum(dout * out), recomputing P from ``lse``."""
        for name, t in (("q", q), ("k", k), ("v", v), ("out", out), ("dout", dout), ("lse", lse)):
            _check_cuda(name, t)
        B, H, Lq, D = q.shape
        Lk = k.shape[2]
        if scale is None:
            scale = 1.0 / math.sqrt(D)
        dq = torch.empty_like(q) if dq is None else dq
        dk = torch.empty_like(k) if dk is None else dk
        dv = torch.empty_like(v) if dv is None else dv
        a = _lib.BwdArgs()
        a.dtype = _dtype_code(q)
        a.batch, a.heads, a.q_len, a.kv_len, a.head_dim = B, H, Lq, Lk, D
        a.head_begin, a.head_count = head_begin, head_count
        a.q, a.k, a.v = _view("q", q, (B, H, Lq, D)), _view("k", k, (B, H, Lk, D)), _view("v", v, (B, H, Lk, D))
        a.out, a.dout = _view("out", out, (B, H, Lq, D)), _view("dout", dout, (B, H, Lq, D))
        if lse.dtype != torch.float32 or tuple(lse.shape) != (B, H, Lq) or lse.stride(2) != 1:
            raise Failure.shape("lse", lse.shape, f"[{B}, {H}, {Lq}] float32")
        a.lse, a.lse_stride_b, a.lse_stride_h = lse.data_ptr(), lse.stride(0), lse.stride(1)
        a.dq, a.dk, a.dv = _view("dq", dq, (B, H, Lq, D)), _view("dk", dk, (B, H, Lk, D)), _view("dv", dv, (B, H, Lk, D))
        a.scale = float(scale)
        if key_mask is not None:
            if tuple(key_mask.shape) != (B, Lk):
                raise Failure.shape("key_mask", key_mask.shape, f"[{B}, {Lk}] bool")
            a.key_mask, a.key_mask_stride_b = key_mask.data_ptr(), key_mask.stride(0)
        a.q_rotary = _rotary("q_rotary", q_rotary, B, H, Lq, D, q.dtype)
        a.k_rotary = _rotary("k_rotary", k_rotary, B, H, Lk, D, q.dtype)
        L = _lib.load()
        ws_bytes = int(L.ltxattn_bwd_workspace(ctypes.byref(a)))
        ws = None
        if ws_bytes > 0:
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
            a.workspace, a.workspace_bytes = ws.data_ptr(), ws_bytes
        rc = L.ltxattn_bwd(ctypes.byref(a), ctypes.c_void_p(_stream_ptr(stream)))
        if rc != _lib.OK:
            raise Failure.from_status(rc)
        return dq, dk, dv


class PreparedAttention:
    """A marshalled ``ltxattn_fwd`` call with its own workspace (see ``AttentionBackend.prepare``)."""

    def __init__(self, args: _lib.FwdArgs, out: torch.Tensor, lse: Optional[torch.Tensor], keep):
        self.args, self.out, self.lse = args, out, lse
        self._keep = keep  # the tensors the argument block points into stay alive
        L = _lib.load()
        n = int(L.ltxattn_fwd_workspace(ctypes.byref(args)))
        self.workspace = torch.empty(max(n, 1), dtype=torch.uint8, device=out.device) if n else None
        if n:
            args.workspace, args.workspace_bytes = self.workspace.data_ptr(), n
        self._fn = L.ltxattn_fwd
        self._ref = ctypes.byref(args)

    def run(self, stream=None):
        rc = self._fn(self._ref, ctypes.c_void_p(_stream_ptr(stream)))
        if rc != _lib.OK:
            raise Failure.from_status(rc)
        return self.out, self.lse


def scaled_dot_product_attention(queries: torch.Tensor, keys: torch.Tensor, values: torch.Tensor,
                                 scale: float, mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``MLXFast.scaledDotProductAttention(queries:keys:values:scale:mask:)``.

    ``mask`` is a boolean key-padding mask ``[B, Lk]`` (True = attend) or None
    (``mask: .none``, DiTAttention.swift:376).
    """
    out, _ = AttentionBackend.attention(queries, keys, values, scale, key_mask=mask)
    return out


def apply_split_rope(x: torch.Tensor, rotary: Rotary, out: Optional[torch.Tensor] = None,
                     stream=None) -> torch.Tensor:
    """``applySplitRoPE(x, rotary)`` (DiTAttention.swift:206-234) through ``ltxattn_rope``.

    ``x`` is a ``[B, heads, tokens, D]`` CUDA view; ``out`` defaults to a new
    tensor and may be ``x`` itself (rotation in place).  In bf16 every product
    and sum rounds to bf16.
    """
    _check_cuda("x", x)
    if x.dim() != 4:
        raise Failure.shape("x", x.shape, "[B, heads, tokens, headDim]")
    B, H, T, D = x.shape
    if out is None:
        out = torch.empty_like(x)
    a = _lib.RopeArgs()
    a.dtype = _dtype_code(x)
    if out.dtype != x.dtype:
        raise Failure("dtype", "out must have the dtype of x", _lib.ERR_DTYPE)
    a.batch, a.heads, a.tokens, a.head_dim = B, H, T, D
    a.x = _view("x", x, (B, H, T, D))
    a.out = _view("out", out, (B, H, T, D))
    a.rotary = _rotary("rotary", rotary, B, H, T, D, x.dtype)
    rc = _lib.load().ltxattn_rope(ctypes.byref(a), ctypes.c_void_p(_stream_ptr(stream)))
    if rc != _lib.OK:
        raise Failure.from_status(rc)
    return out


def rotary_tables(positions: torch.Tensor, max_pos, inner: int, heads: int, theta: float = 10000.0,
                  dtype=torch.bfloat16, stream=None) -> Rotary:
    """``DiTForward.rotary`` (DiTForward.swift:641-678) on the device through ``ltxattn_rotary_tables``.

    ``positions`` is a CUDA float32 tensor ``[n_pos, tokens, 2]`` of (lo, hi)
    bounds; returns per-head tables ``[1, heads, tokens, inner/2/heads]``.
    """
    _check_cuda("positions", positions)
    if positions.dtype != torch.float32 or positions.dim() != 3 or positions.shape[2] != 2:
        raise Failure.shape("positions", positions.shape, "[n_pos, tokens, 2] float32")
    positions = positions.contiguous()
    n_pos, tokens, _ = positions.shape
    per = inner // 2 // heads if heads > 0 else 0
    cos = torch.empty((1, heads, tokens, per), dtype=dtype, device=positions.device)
    sin = torch.empty_like(cos)
    a = _lib.RotaryTableArgs()
    a.dtype = _dtype_code(cos)
    a.n_pos, a.tokens, a.inner, a.heads, a.theta = n_pos, tokens, inner, heads, float(theta)
    for d, v in enumerate(list(max_pos)[:4]):
        a.max_pos[d] = float(v)
    a.positions, a.cos, a.sin = positions.data_ptr(), cos.data_ptr(), sin.data_ptr()
    rc = _lib.load().ltxattn_rotary_tables(ctypes.byref(a), ctypes.c_void_p(_stream_ptr(stream)))
    if rc != _lib.OK:
        raise Failure.from_status(rc)
    return Rotary(cos, sin)


def _qk_args(x: torch.Tensor, weight: torch.Tensor, heads: int, rotary: Optional[Rotary], eps: float,
             out: Optional[torch.Tensor]):
    _check_cuda("x", x)
    if x.dim() != 3 or x.stride(2) != 1 or x.shape[2] % heads:
        raise Failure.shape("x", x.shape, f"[B, tokens, {heads} * headDim] with a unit last stride")
    B, T, inner = x.shape
    D = inner // heads
    if out is None:
        out = torch.empty((B, heads, T, D), dtype=x.dtype, device=x.device)
    _check_cuda("weight", weight)
    if weight.dtype != x.dtype or tuple(weight.shape) != (inner,) or not weight.is_contiguous():
        raise Failure.shape("weight", weight.shape, f"[{inner}] contiguous, dtype {x.dtype}")
    a = _lib.QkPrepArgs()
    a.dtype = _dtype_code(x)
    a.batch, a.tokens, a.heads, a.head_dim = B, T, heads, D
    a.x, a.x_stride_b, a.x_stride_t = x.data_ptr(), x.stride(0), x.stride(1)
    a.weight, a.eps = weight.data_ptr(), float(eps)
    a.rotary = _rotary("rotary", rotary, B, heads, T, D, x.dtype)
    a.out = _view("out", out, (B, heads, T, D))
    return a, out


def qk_prep(x: torch.Tensor, weight: torch.Tensor, heads: int, rotary: Optional[Rotary] = None,
            eps: float = 1e-6, out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """q / k preparation of ``DiTAttention`` (DiTAttention.swift:358-367) through ``ltxattn_qk_prep``.

    ``x`` is the projection output ``[B, tokens, heads * D]`` (unit stride along
    the last dim); returns ``split-RoPE(split(rmsNorm(x, weight)))`` as
    ``[B, heads, tokens, D]`` (or into ``out``).
    """
    a, out = _qk_args(x, weight, heads, rotary, eps, out)
    rc = _lib.load().ltxattn_qk_prep(ctypes.byref(a), ctypes.c_void_p(_stream_ptr(stream)))
    if rc != _lib.OK:
        raise Failure.from_status(rc)
    return out


def qk_prep_pair(xq: torch.Tensor, wq: torch.Tensor, xk: torch.Tensor, wk: torch.Tensor, heads: int,
                 q_rotary: Optional[Rotary] = None, k_rotary: Optional[Rotary] = None, eps: float = 1e-6,
                 out_q: Optional[torch.Tensor] = None, out_k: Optional[torch.Tensor] = None, stream=None):
    """``qk_prep`` of q and of k in one launch (``ltxattn_qk_prep_pair``); returns ``(qh, kh)``.
    The key stream may have its own token count (a cross-attention)."""
    aq, out_q = _qk_args(xq, wq, heads, q_rotary, eps, out_q)
    ak, out_k = _qk_args(xk, wk, heads, k_rotary, eps, out_k)
    rc = _lib.load().ltxattn_qk_prep_pair(ctypes.byref(aq), ctypes.byref(ak), ctypes.c_void_p(_stream_ptr(stream)))
    if rc != _lib.OK:
        raise Failure.from_status(rc)
    return out_q, out_k


def device_status(clear: bool = True) -> int:
    """Status of the current device's kernel error word (synchronises)."""
    site = ctypes.c_int32(0)
    return int(_lib.load().ltxattn_device_status(int(clear), ctypes.byref(site)))


def device_info(device: int = 0) -> dict:
    info = _lib.DeviceInfo()
    rc = _lib.load().ltxattn_device_query(device, ctypes.byref(info))
    if rc != _lib.OK:
        raise Failure.from_status(rc)
    return {f: (getattr(info, f).decode() if f == "name" else getattr(info, f)) for f, _ in info._fields_}
