"""Seeded synthetic inputs for the attention configurations.

Input preparation only (no attention arithmetic): a counter-based splitmix64
stream into fp64 Box-Muller, per-head RMSNorm with unit weight, bf16
round-to-nearest-even, and the RoPE tables the benchmark configurations name.

* splitmix64 is the generator of ``Sources/ltx/Bench.swift:479-493``; the
  per-tensor seed offsets (q: +2, k: +3, v: +4, dO: +5) mirror
  ``Sources/ltx/BenchGEMM.swift:627-632``.
* Split-RoPE tables are ``[1, Ht, T, D/2]`` (cos, sin), the layout of
  ``DiTAttention.Rotary`` (``DiTAttention.swift:92-105``).
* ``reference_rotary`` restates ``DiTForward.rotary`` /
  ``frequencyGrid`` / ``videoPositions`` / ``audioPositions``
  (``Sources/LTXModules/DiTForward.swift:455-466,486-519,606-619,641-678``).
"""
from __future__ import annotations

import math

import numpy as np

GOLDEN = np.uint64(0x9E3779B97F4A7C15)
M1 = np.uint64(0xBF58476D1CE4E5B9)
M2 = np.uint64(0x94D049BB133111EB)

SEED_OFFSETS = {"q": 2, "k": 3, "v": 4, "dout": 5}


def _splitmix64_at(seed: int, idx: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + GOLDEN * (idx + np.uint64(1))
        z = (z ^ (z >> np.uint64(30))) * M1
        z = (z ^ (z >> np.uint64(27))) * M2
        return z ^ (z >> np.uint64(31))


def normal(seed: int, n: int, chunk: int = 1 << 22, start: int = 0) -> np.ndarray:
    """Draws start .. start+n-1 of N(0,1) as float32; element i depends only on (seed, i)."""
    out = np.empty(n, dtype=np.float32)
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        i = np.arange(start + s, start + e, dtype=np.uint64)
        a = _splitmix64_at(seed, np.uint64(2) * i)
        b = _splitmix64_at(seed, np.uint64(2) * i + np.uint64(1))
        u1 = ((a >> np.uint64(11)).astype(np.float64) + 1.0) * 2.0 ** -53
        u2 = (b >> np.uint64(11)).astype(np.float64) * 2.0 ** -53
        out[s:e] = (np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * math.pi * u2)).astype(np.float32)
    return out


def bench_bits(seed: int, n: int) -> np.ndarray:
    """The reference bench's operands (``BenchOperand.bits``,
    ``Sources/ltx/Bench.swift:474-493``): a sequential splitmix64 stream whose
    state starts at seed + golden and advances by golden before each draw; the
    top 24 bits of each output as a unit in [0, 1), centred to (unit - 0.5) * 2
    and rounded to bf16.  Returned as float32 values (exactly the bf16 ones)."""
    i = np.arange(n, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + GOLDEN * (i + np.uint64(2))
        z = (z ^ (z >> np.uint64(30))) * M1
        z = (z ^ (z >> np.uint64(27))) * M2
        z = z ^ (z >> np.uint64(31))
    unit = (z >> np.uint64(40)).astype(np.float32) / np.float32(1 << 24)
    return round_bf16((unit - np.float32(0.5)) * np.float32(2.0))


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns (uint16), round to nearest even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7F800000) == 0x7F800000
    r = ((u >> 16) & 1) + np.uint32(0x7FFF)
    with np.errstate(over="ignore"):
        rounded = ((u + r) >> 16).astype(np.uint16)
    keep = (u >> 16).astype(np.uint16)
    return np.where(nan, keep, rounded)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    return bf16_to_f32(bf16_bits(x))


def rms_norm_heads(x: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """Per-head RMSNorm over the last dim with unit weight, fp32 statistics."""
    x = x.astype(np.float32)
    ms = np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True).astype(np.float32)
    return (x * (1.0 / np.sqrt(ms + np.float32(eps))).astype(np.float32)).astype(np.float32)


def seeded_tensor(seed: int, shape, *, rmsnorm: bool = False, bf16: bool = True, heads=None) -> np.ndarray:
    """A float32 array holding exactly the values the device receives.

    ``heads=(h0, hc)`` with a [B, H, T, D] shape gives heads h0 .. h0+hc-1 of
    that tensor, the same values as slicing the whole one (how a rank of a
    head-sharded job builds only its own block)."""
    if heads is None:
        n = int(np.prod(shape))
        x = normal(seed, n).reshape(shape)
    else:
        B, H, T, D = shape
        h0, hc = heads
        if not (0 <= h0 and hc >= 1 and h0 + hc <= H):
            raise ValueError(f"heads {heads} outside [0, {H})")
        per = T * D
        x = np.stack([normal(seed, hc * per, start=(b * H + h0) * per).reshape(hc, T, D) for b in range(B)])
    if rmsnorm:
        x = rms_norm_heads(x)
    if bf16:
        x = round_bf16(x)
    return x


# --------------------------------------------------------------------------
# RoPE tables for the benchmark configurations


def _tables_from_angles(angles: np.ndarray, bf16: bool):
    cos = np.cos(angles.astype(np.float64)).astype(np.float32)
    sin = np.sin(angles.astype(np.float64)).astype(np.float32)
    if bf16:
        cos, sin = round_bf16(cos), round_bf16(sin)
    return cos[None, None], sin[None, None]


def rope3d_grid(frames: int, height: int, width: int, head_dim: int,
                theta: float = 10000.0, bf16: bool = True):
    """3D split-RoPE over an integer (t, h, w) grid, shared by all heads.

    The head's D/2 rotary pairs are one leading identity pair (the reference
    pads at the front, DiTForward.swift:666-672) followed by three equal
    bands for t, h and w with inverse frequencies theta^(-j/n), j < n.
    Returns (cos, sin) of shape [1, 1, T, D/2], T = frames*height*width,
    tokens ordered (t, h, w) with w fastest (DiTForward.swift:484-485).
    """
    half = head_dim // 2
    n = (half - 1) // 3
    pad = half - 3 * n
    inv = theta ** (-np.arange(n, dtype=np.float64) / n)
    t, h, w = np.meshgrid(np.arange(frames), np.arange(height), np.arange(width), indexing="ij")
    pos = np.stack([t.ravel(), h.ravel(), w.ravel()], axis=-1).astype(np.float64)
    ang = np.concatenate([np.zeros((pos.shape[0], pad))] +
                         [pos[:, i:i + 1] * inv[None, :] for i in range(3)], axis=-1)
    return _tables_from_angles(ang, bf16)


def rope1d(positions: np.ndarray, head_dim: int, theta: float = 10000.0, bf16: bool = True):
    """1D split-RoPE: angle = position * theta^(-j/(D/2)), j < D/2."""
    half = head_dim // 2
    inv = theta ** (-np.arange(half, dtype=np.float64) / half)
    ang = np.asarray(positions, dtype=np.float64)[:, None] * inv[None, :]
    return _tables_from_angles(ang, bf16)


def video_frame_seconds(frames: int, tokens_per_frame: int, temporal_scale: int = 8,
                        fps: float = 24.0) -> np.ndarray:
    """Each video token's time: centre of its latent frame's causal pixel span.

    Latent frame t covers pixel frames [max(8t-7, 0), 8t+1) (the causal
    correction of DiTForward.swift:501-511), divided by the frame rate.
    """
    t = np.arange(frames)
    lo = np.maximum(t * temporal_scale + 1 - temporal_scale, 0) / fps
    hi = np.maximum((t + 1) * temporal_scale + 1 - temporal_scale, 0) / fps
    return np.repeat((lo + hi) / 2.0, tokens_per_frame)


def audio_token_seconds(tokens: int, hop: int = 160, sample_rate: int = 16000,
                        downsample: int = 4) -> np.ndarray:
    """Audio token centres in seconds (DiTForward.swift:606-619)."""
    def sec(i):
        frame = np.maximum(np.asarray(i, np.float64) * downsample + 1 - downsample, 0)
        return frame * hop / sample_rate
    i = np.arange(tokens)
    return (sec(i) + sec(i + 1)) / 2.0


# --------------------------------------------------------------------------
# Restatement of the reference's own table builder (per-head distinct tables)


def frequency_grid(theta: float, n_pos: int, inner: int) -> np.ndarray:
    """DiTForward.frequencyGrid (:455-466): fp64 linspace exponent, fp32 out."""
    count = inner // (2 * n_pos)
    step = 1.0 / (count - 1)
    vals = np.empty(count, dtype=np.float32)
    for i in range(count):
        e = 1.0 if i == count - 1 else i * step
        vals[i] = np.float32(math.pow(theta, e) * math.pi / 2)
    return vals


def video_positions(frames: int, height: int, width: int, temporal_scale: int = 8,
                    spatial_scale: int = 32, fps: float = 24.0) -> np.ndarray:
    """DiTForward.videoPositions (:486-519): [3, tokens, 2] pixel bounds, time in s."""
    t, y, x = np.meshgrid(np.arange(frames), np.arange(height), np.arange(width), indexing="ij")
    starts = [t.ravel(), y.ravel(), x.ravel()]
    scales = [temporal_scale, spatial_scale, spatial_scale]
    out = np.empty((3, starts[0].size, 2), np.float32)
    for d in range(3):
        lo = starts[d] * scales[d]
        hi = (starts[d] + 1) * scales[d]
        if d == 0:
            lo = np.maximum(lo + 1 - temporal_scale, 0)
            hi = np.maximum(hi + 1 - temporal_scale, 0)
        lo_f, hi_f = lo.astype(np.float32), hi.astype(np.float32)
        if d == 0:
            lo_f, hi_f = lo_f / np.float32(fps), hi_f / np.float32(fps)
        out[d, :, 0], out[d, :, 1] = lo_f, hi_f
    return out


def audio_positions(tokens: int, hop: int = 160, sample_rate: int = 16000,
                    downsample: int = 4) -> np.ndarray:
    """DiTForward.audioPositions (:606-619): [1, tokens, 2] seconds."""
    def sec(i):
        f = np.maximum(np.float32(i * downsample) + np.float32(1 - downsample), np.float32(0))
        return f * np.float32(hop) / np.float32(sample_rate)
    out = np.empty((1, tokens, 2), np.float32)
    for i in range(tokens):
        out[0, i, 0], out[0, i, 1] = sec(i), sec(i + 1)
    return out


def reference_rotary(positions: np.ndarray, inner: int, max_pos, heads: int,
                     theta: float = 10000.0, bf16: bool = True):
    """DiTForward.rotary (:641-678): per-head tables [1, heads, T, inner/2/heads]."""
    n_pos, tokens, _ = positions.shape
    middle = (positions[:, :, 0] + positions[:, :, 1]) / np.float32(2.0)
    frac = np.stack([middle[d] / np.float32(max_pos[d]) for d in range(n_pos)], axis=-1)
    idx = frequency_grid(theta, n_pos, inner)
    ang = idx[None, None, :] * (frac[:, :, None] * np.float32(2.0) - np.float32(1.0))
    ordered = ang.transpose(0, 2, 1).reshape(tokens, idx.size * n_pos).astype(np.float32)
    cos, sin = np.cos(ordered).astype(np.float32), np.sin(ordered).astype(np.float32)
    pad = inner // 2 - ordered.shape[-1]
    if pad > 0:
        cos = np.concatenate([np.ones((tokens, pad), np.float32), cos], axis=-1)
        sin = np.concatenate([np.zeros((tokens, pad), np.float32), sin], axis=-1)
    per = inner // 2 // heads
    cos = cos.reshape(tokens, heads, per).transpose(1, 0, 2)[None]
    sin = sin.reshape(tokens, heads, per).transpose(1, 0, 2)[None]
    if bf16:
        cos, sin = round_bf16(cos), round_bf16(sin)
    return np.ascontiguousarray(cos), np.ascontiguousarray(sin)
