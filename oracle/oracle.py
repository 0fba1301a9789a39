"""ctypes front end of the CPU restatement in ``ltxattn_oracle.c``.

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, by ``__graft_entry__.smoke()``
as the checker, and by ``bench.py``'s CPU-baseline leg.  The product library
(``libltxattn_cuda``) never loads it.

Every function takes and returns numpy float32 arrays in contiguous
``[B, H, T, D]`` layout (see the C file's header for the reference lines each
one restates).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libltxattn_oracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)


def build() -> str:
    """Compile the oracle with the Makefile beside this file."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        src = os.path.join(_HERE, "ltxattn_oracle.c")
        if (not os.path.exists(_LIB_PATH)
                or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src)):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.oracle_fill_normal.argtypes = [ctypes.c_uint64, ctypes.c_int64, _f32p]
        L.oracle_round_bf16.argtypes = [_f32p, ctypes.c_int64]
        L.oracle_rope.argtypes = [_f32p, _f32p, _f32p] + [ctypes.c_int] * 4 + [
            ctypes.c_int64, ctypes.c_int64, ctypes.c_int]
        L.oracle_rope_bwd.argtypes = L.oracle_rope.argtypes
        L.oracle_attn_fwd.argtypes = [_f32p, _f32p, _f32p, _u8p, ctypes.c_int64] + [
            ctypes.c_int] * 5 + [ctypes.c_double, _f32p, _f32p, ctypes.c_int]
        L.oracle_attn_fwd_f32.argtypes = [_f32p, _f32p, _f32p, _u8p, ctypes.c_int64] + [
            ctypes.c_int] * 5 + [ctypes.c_float, _f32p, _f32p, ctypes.c_int]
        L.oracle_attn_bwd.argtypes = [_f32p, _f32p, _f32p, _u8p, ctypes.c_int64, _f32p] + [
            ctypes.c_int] * 5 + [ctypes.c_double, _f32p, _f32p, _f32p, ctypes.c_int]
        L.oracle_rotary_tables.argtypes = [_f32p, _f32p] + [ctypes.c_int] * 4 + [ctypes.c_double, _f32p, _f32p]
        L.oracle_attn_fwd_gemma.argtypes = [_f32p, _f32p, _f32p, _u8p] + [ctypes.c_int] * 5 + [
            ctypes.c_double, ctypes.c_int, ctypes.c_int, _f32p, _f32p]
        L.oracle_qk_prep.argtypes = [_f32p, _f32p] + [ctypes.c_int] * 4 + [ctypes.c_float, _f32p, _f32p,
                                                                         ctypes.c_int64, ctypes.c_int64,
                                                                         ctypes.c_int, _f32p]
        L.oracle_attn_bwd_keys.argtypes = [_f32p] * 6 + [ctypes.c_int] * 3 + [
            ctypes.c_double, ctypes.POINTER(ctypes.c_int), ctypes.c_int, _f32p, _f32p, ctypes.c_int]
        L.oracle_attn_bwd_keys.restype = ctypes.c_int
        for f in ("oracle_rope", "oracle_rope_bwd", "oracle_attn_fwd",
                  "oracle_attn_fwd_f32", "oracle_attn_bwd", "oracle_rotary_tables", "oracle_qk_prep",
                  "oracle_attn_fwd_gemma"):
            getattr(L, f).restype = ctypes.c_int
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data_as(_f32p)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def fill_normal(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().oracle_fill_normal(ctypes.c_uint64(seed), n, _p(out))
    return out


def round_bf16(x: np.ndarray) -> np.ndarray:
    y = _f32(x).copy()
    lib().oracle_round_bf16(_p(y), y.size)
    return y


def _table_strides(tab: np.ndarray, H: int):
    """Tables are [Bt, Ht, T, D/2]; Bt, Ht in {1, B/H}.  Size-1 dims get stride 0."""
    Bt, Ht, T, half = tab.shape
    sb = 0 if Bt == 1 else Ht * T * half
    sh = 0 if Ht == 1 else T * half
    return sb, sh


def rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, bf16: bool) -> np.ndarray:
    y = _f32(x).copy()
    B, H, T, D = y.shape
    c, s = _f32(cos), _f32(sin)
    sb, sh = _table_strides(c, H)
    rc = lib().oracle_rope(_p(y), _p(c), _p(s), B, H, T, D, sb, sh, int(bf16))
    assert rc == 0
    return y


def rope_bwd(dx: np.ndarray, cos: np.ndarray, sin: np.ndarray, bf16_tables: bool) -> np.ndarray:
    y = _f32(dx).copy()
    B, H, T, D = y.shape
    c, s = _f32(cos), _f32(sin)
    sb, sh = _table_strides(c, H)
    rc = lib().oracle_rope_bwd(_p(y), _p(c), _p(s), B, H, T, D, sb, sh, int(bf16_tables))
    assert rc == 0
    return y


def _mask_args(mask, B, Lk):
    if mask is None:
        return None, 0, None
    m = np.ascontiguousarray(mask, dtype=np.uint8).reshape(B, Lk)
    return m.ctypes.data_as(_u8p), Lk, m


def attn_fwd(q, k, v, mask=None, scale=None, threads=0):
    """fp64-accumulated forward; returns (out[B,H,Lq,D], lse[B,H,Lq])."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    B, H, Lq, D = q.shape
    Lk = k.shape[2]
    if scale is None:
        scale = 1.0 / np.sqrt(D)
    out = np.empty((B, H, Lq, D), np.float32)
    lse = np.empty((B, H, Lq), np.float32)
    mp, ms, _keep = _mask_args(mask, B, Lk)
    rc = lib().oracle_attn_fwd(_p(q), _p(k), _p(v), mp, ms, B, H, Lq, Lk, D,
                               float(scale), _p(out), _p(lse), threads)
    assert rc == 0
    return out, lse


def attn_fwd_f32(q, k, v, mask=None, scale=None, threads=0):
    """fp32 explicit-path forward (the timed CPU baseline)."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    B, H, Lq, D = q.shape
    Lk = k.shape[2]
    if scale is None:
        scale = 1.0 / np.sqrt(D)
    out = np.empty((B, H, Lq, D), np.float32)
    lse = np.empty((B, H, Lq), np.float32)
    mp, ms, _keep = _mask_args(mask, B, Lk)
    rc = lib().oracle_attn_fwd_f32(_p(q), _p(k), _p(v), mp, ms, B, H, Lq, Lk, D,
                                   float(scale), _p(out), _p(lse), threads)
    assert rc == 0
    return out, lse


def attn_bwd(q, k, v, dout, mask=None, scale=None, threads=0):
    """fp64-accumulated backward w.r.t. the (rotated) q, k and v."""
    q, k, v, dout = _f32(q), _f32(k), _f32(v), _f32(dout)
    B, H, Lq, D = q.shape
    Lk = k.shape[2]
    if scale is None:
        scale = 1.0 / np.sqrt(D)
    dq = np.empty_like(q)
    dk = np.empty_like(k)
    dv = np.empty_like(v)
    mp, ms, _keep = _mask_args(mask, B, Lk)
    rc = lib().oracle_attn_bwd(_p(q), _p(k), _p(v), mp, ms, _p(dout), B, H, Lq, Lk, D,
                               float(scale), _p(dq), _p(dk), _p(dv), threads)
    assert rc == 0
    return dq, dk, dv


def attn_bwd_keys(q, k, v, dout, lse, delta, keys, scale=None, threads=0):
    """dK, dV of the key indices ``keys`` of one unmasked head ([Lq, D] / [Lk, D]
    arrays), streaming over query rows; ``lse`` and ``delta`` = rowsum(dout * out)
    come from a forward of the same head.  Returns (dk, dv) as [len(keys), D]."""
    q, k, v, dout = _f32(q), _f32(k), _f32(v), _f32(dout)
    lse, delta = _f32(lse).reshape(-1), _f32(delta).reshape(-1)
    Lq, D = q.shape
    Lk = k.shape[0]
    if scale is None:
        scale = 1.0 / np.sqrt(D)
    idx = np.ascontiguousarray(keys, dtype=np.int32)
    dk = np.empty((idx.size, D), np.float32)
    dv = np.empty((idx.size, D), np.float32)
    rc = lib().oracle_attn_bwd_keys(_p(q), _p(k), _p(v), _p(dout), _p(lse), _p(delta), Lq, Lk, D, float(scale),
                                    idx.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), idx.size, _p(dk), _p(dv),
                                    threads)
    assert rc == 0
    return dk, dv


def attention_reference(q, k, v, mask=None, q_rot=None, k_rot=None, bf16=False, scale=None):
    """Full reference composition: RoPE (:364-367) then SDPA (:369-382).

    ``q_rot`` / ``k_rot`` are ``(cos, sin)`` pairs or None; ``k_rot`` None with
    ``q_rot`` given means "use the query's table for the key", as
    ``keyRotary ?? rotary`` does at DiTAttention.swift:366.
    """
    if q_rot is not None:
        if k_rot is None:
            k_rot = q_rot
        q = rope(q, q_rot[0], q_rot[1], bf16)
        k = rope(k, k_rot[0], k_rot[1], bf16)
    return attn_fwd(q, k, v, mask=mask, scale=scale)


if __name__ == "__main__":  # pragma: no cover
    print(build())


def rotary_tables(positions: np.ndarray, max_pos, inner: int, heads: int, theta: float = 10000.0):
    """DiTForward.rotary restated in C: fp32 tables [1, heads, tokens, inner/2/heads]."""
    pos = _f32(positions)
    n_pos, tokens, _ = pos.shape
    mp = np.asarray(max_pos, dtype=np.float32)
    per = inner // 2 // heads
    c = np.empty((heads, tokens, per), np.float32)
    s = np.empty_like(c)
    rc = lib().oracle_rotary_tables(_p(pos), _p(mp), n_pos, tokens, inner, heads, float(theta), _p(c), _p(s))
    assert rc == 0
    return c[None], s[None]


def qk_prep(x: np.ndarray, w: np.ndarray, heads: int, eps: float = 1e-6, cos=None, sin=None,
            bf16: bool = True) -> np.ndarray:
    """DiTAttention q/k preparation restated in C: rmsNorm over the inner dim, head
    split, split RoPE.  x [B, T, inner] -> [B, heads, T, inner / heads]."""
    xx = _f32(x)
    B, T, inner = xx.shape
    D = inner // heads
    out = np.empty((B, heads, T, D), np.float32)
    c = s = None
    sb = sh = 0
    if cos is not None:
        c, s = _f32(cos), _f32(sin)
        sb, sh = _table_strides(c, heads)
    null = ctypes.POINTER(ctypes.c_float)()
    rc = lib().oracle_qk_prep(_p(xx), _p(_f32(w)), B, T, heads, D, float(eps),
                              _p(c) if c is not None else null, _p(s) if s is not None else null,
                              sb, sh, int(bf16), _p(out))
    assert rc == 0
    return out


def attention_gemma(q, k, v, valid=None, scale=1.0, causal=True, window=0):
    """Gemma text-encoder self-attention (causal / sliding / padding masks with the
    un-masking of empty rows, grouped KV heads), fp64: returns (out, lse)."""
    qq, kk, vv = _f32(q), _f32(k), _f32(v)
    B, Hq, L, D = qq.shape
    Hkv = kk.shape[1]
    out = np.empty_like(qq)
    lse = np.empty((B, Hq, L), np.float32)
    m = np.ascontiguousarray(valid, dtype=np.uint8) if valid is not None else None
    mp = m.ctypes.data_as(_u8p) if m is not None else ctypes.POINTER(ctypes.c_uint8)()
    rc = lib().oracle_attn_fwd_gemma(_p(qq), _p(kk), _p(vv), mp, B, Hq, Hkv, L, D, float(scale),
                                     int(causal), int(window), _p(out), _p(lse))
    assert rc == 0
    return out, lse


def gate_value(logits, bf16=True):
    """The per-head gate 2 * sigmoid(logit) of DiTAttention.swift:395-396: the
    sigmoid in fp32 and cast back to the activation dtype (:240-242; here fp64
    rounded to fp32, then to bf16 for bf16 activations), then the exact doubling."""
    x = _f32(logits).astype(np.float64)
    s = (1.0 / (1.0 + np.exp(-x))).astype(np.float32)
    if bf16:
        s = round_bf16(s)
    return (2.0 * s).astype(np.float32)


def gate_output(out, logits, bf16=True):
    """out [B, H, T, D] (values in the activation dtype) times the gate of
    logits [B, T, H], broadcast over D and rounded to the activation dtype
    (DiTAttention.swift:397-399: `out * gates.transposed(0, 2, 1)[..., None]`)."""
    g = gate_value(logits, bf16).transpose(0, 2, 1)[..., None]
    y = (_f32(out).astype(np.float64) * g.astype(np.float64)).astype(np.float32)
    return round_bf16(y) if bf16 else y


def linear(x, weight, bias=None):
    """DiTAttention.linear (DiTAttention.swift:178-188) for bf16 activations: the
    matmul x W^T (accumulated here in fp64) rounded to bf16, then the bias added
    and rounded again -- the reference's two roundings."""
    y = round_bf16(_f32(x).astype(np.float64) @ _f32(weight).astype(np.float64).T)
    if bias is not None:
        y = round_bf16(y.astype(np.float64) + _f32(bias).astype(np.float64))
    return y


def dit_attention_module(x, w, heads, cos=None, sin=None, k_cos=None, k_sin=None, context=None):
    """DiTAttention.callAsFunction (DiTAttention.swift:315-404) for bf16
    activations, on the CPU: every projection is an fp64 matmul rounded to bf16
    plus a bf16-rounded bias add (:178-189); q and k take ``qk_prep`` (rmsNorm
    over the inner dim, split, split RoPE with ``k_cos/k_sin`` or else the q
    tables for k, :358-367); the attention is ``attn_fwd`` rounded to bf16; the
    gate (when ``to_gate_logits.weight`` is present) ``gate_output``; then the
    merge and ``to_out.0``.  ``w`` maps checkpoint names without the block
    prefix to float32 arrays holding bf16 values."""
    def lin(a, name):
        return linear(a, w[name + ".weight"], w.get(name + ".bias"))
    kv = x if context is None else context
    B, T, _ = x.shape
    Tk = kv.shape[1]
    inner = w["to_q.weight"].shape[0]
    D = inner // heads
    v = lin(kv, "to_v")
    q = qk_prep(lin(x, "to_q"), w["q_norm.weight"], heads, 1e-6, cos, sin, bf16=True)
    kc, ks = (k_cos, k_sin) if k_cos is not None else (cos, sin)
    k = qk_prep(lin(kv, "to_k"), w["k_norm.weight"], heads, 1e-6, kc, ks, bf16=True)
    vh = np.ascontiguousarray(v.reshape(B, Tk, heads, D).transpose(0, 2, 1, 3))
    out, _ = attn_fwd(q, k, vh)
    out = round_bf16(out)
    if "to_gate_logits.weight" in w:
        out = gate_output(out, lin(x, "to_gate_logits"), True)
    merged = np.ascontiguousarray(out.transpose(0, 2, 1, 3).reshape(B, T, inner))
    return lin(merged, "to_out.0")
