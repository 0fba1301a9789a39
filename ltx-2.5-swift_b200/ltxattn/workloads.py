"""The benchmark configurations: shapes, rotary tables, masks and inputs.

BASELINE configurations 2-5 of the fused attention (config 1 is the fp32
parity gate of the tests), the reference-faithful 101-token audio stream
(``Sources/LTXFoundation/LatentGeometry.swift:129-132``: round(97 / 24 * 25))
and the attention case set of the reference's own ``ltx bench gemm``
(``Sources/ltx/BenchGEMM.swift:466-497``, operands from
``BenchOperand.bits``, ``Sources/ltx/Bench.swift:474-493``).

Inputs are host arrays holding exactly the values the device receives.
``heads=(h0, hc)`` builds only heads h0 .. h0+hc-1 of the whole tensor, which
is how a rank of a head-sharded job makes its block: the blocks of all ranks
together are the single-GPU job.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import numpy as np

from . import inputs


@dataclass(frozen=True)
class Workload:
    name: str
    B: int
    H: int
    Lq: int
    Lk: int
    D: int
    rope: Optional[str]      # None, "3d" (video grid), "1d" (token index), "av" / "va" (shared seconds clock)
    mask_valid: Optional[int]  # keys [0, mask_valid) valid, or None for no mask
    rms: bool                # per-head RMSNorm of q and k (BASELINE's input recipe)
    bound: str               # "tensor" or "hbm": the roofline of the attention kernel
    desc: str

    @property
    def flops(self) -> float:
        """4 B H Lq Lk D, the reference's convention (BenchGEMM.swift:289)."""
        return 4.0 * self.B * self.H * self.Lq * self.Lk * self.D

    @property
    def effective_flops(self) -> float:
        return 4.0 * self.B * self.H * self.Lq * (self.mask_valid or self.Lk) * self.D

    def algorithmic_bytes(self, heads: Optional[int] = None) -> float:
        """Bytes one attention call must move: Q and O, plus K and V of the valid keys (bf16)."""
        h = self.H if heads is None else heads
        valid = self.mask_valid or self.Lk
        return 2.0 * (2 * self.B * h * self.Lq * self.D + 2 * self.B * h * valid * self.D)


WORKLOADS = {
    "c2": Workload("c2", 1, 32, 3120, 3120, 128, "3d", None, True, "tensor",
                   "video self-attn 640x384x97, 3120 tok, H32 D128, 3D RoPE"),
    "c3": Workload("c3", 1, 32, 3120, 1024, 128, None, 94, True, "hbm",
                   "text cross-attn Q3120 x KV1024 (94 valid), H32 D128"),
    "c4a": Workload("c4a", 1, 32, 126, 126, 64, "1d", None, True, "hbm",
                    "audio self-attn 126 tok, H32 D64, 1D RoPE"),
    "c4b": Workload("c4b", 1, 32, 3120, 126, 64, "av", None, True, "hbm",
                    "video->audio cross Q3120 x KV126, H32 D64, time RoPE"),
    "c4c": Workload("c4c", 1, 32, 126, 3120, 64, "va", None, True, "hbm",
                    "audio->video cross Q126 x KV3120, H32 D64, time RoPE"),
    "c5": Workload("c5", 1, 32, 29760, 29760, 128, None, None, False, "tensor",
                   "video self-attn 1280x768x241, 29760 tok, H32 D128"),
    "a101": Workload("a101", 1, 32, 101, 101, 64, "1d", None, True, "hbm",
                     "audio self-attn at the reference's 101 audio tokens (97 frames), H32 D64, 1D RoPE"),
}

# BenchGEMM.swift:466-497 at the 640x384x97 geometry: 32 heads, video width 4096
# (D 128), audio width 2048 (D 64), 3120 video tokens, 101 audio tokens, 1024
# text tokens; no mask, no RoPE, scale 1/sqrt(D).
BENCH_GEMM_CASES = (
    ("attn1.video_self", 3120, 3120, 128),
    ("audio_attn1.audio_self", 101, 101, 64),
    ("attn2.video_text_cross", 3120, 1024, 128),
    ("audio_attn2.audio_text_cross", 101, 1024, 64),
    ("audio_to_video_attn.cross", 3120, 101, 64),
    ("video_to_audio_attn.cross", 101, 3120, 64),
)
BENCH_GEMM_SEED = 0x5EED  # BenchGEMM.swift:119; q, k, v take seed + 2, 3, 4 (:627-632)
DEFAULT_SEED = 1000


def tables(w: Workload) -> Optional[Tuple[Tuple[np.ndarray, np.ndarray], Optional[Tuple[np.ndarray, np.ndarray]]]]:
    """(q table, k table or None = the q table) as bf16-valued (cos, sin) arrays [1, 1, T, D/2]."""
    if w.rope == "3d":
        return inputs.rope3d_grid(13, 12, 20, w.D), None
    if w.rope == "1d":
        return inputs.rope1d(np.arange(w.Lq, dtype=np.float64), w.D), None
    if w.rope == "av":
        return (inputs.rope1d(inputs.video_frame_seconds(13, 240), w.D),
                inputs.rope1d(inputs.audio_token_seconds(w.Lk), w.D))
    if w.rope == "va":
        return (inputs.rope1d(inputs.audio_token_seconds(w.Lq), w.D),
                inputs.rope1d(inputs.video_frame_seconds(13, 240), w.D))
    return None


def key_mask(w: Workload) -> Optional[np.ndarray]:
    if w.mask_valid is None:
        return None
    m = np.zeros((w.B, w.Lk), np.uint8)
    m[:, :w.mask_valid] = 1
    return m


def host_inputs(w: Workload, heads: Optional[Tuple[int, int]] = None, seed: int = DEFAULT_SEED):
    """q, k, v (float32 arrays of bf16 values, [B, hc, T, D]), tables, mask."""
    hs = heads if heads is not None else (0, w.H)
    q = inputs.seeded_tensor(seed + 2, (w.B, w.H, w.Lq, w.D), rmsnorm=w.rms, heads=hs)
    k = inputs.seeded_tensor(seed + 3, (w.B, w.H, w.Lk, w.D), rmsnorm=w.rms, heads=hs)
    v = inputs.seeded_tensor(seed + 4, (w.B, w.H, w.Lk, w.D), heads=hs)
    return q, k, v, tables(w), key_mask(w)


def host_dout(w: Workload, heads: Optional[Tuple[int, int]] = None, seed: int = DEFAULT_SEED) -> np.ndarray:
    hs = heads if heads is not None else (0, w.H)
    return inputs.seeded_tensor(seed + 5, (w.B, w.H, w.Lq, w.D), heads=hs)


def bench_gemm_inputs(Lq: int, Lk: int, D: int, heads: int = 32, seed: int = BENCH_GEMM_SEED,
                      head_range: Optional[Tuple[int, int]] = None):
    """q, k, v of one BenchGEMM attention case: the reference's operand stream
    over [1, heads, T, D], optionally only heads h0 .. h0+hc-1."""
    h0, hc = head_range if head_range is not None else (0, heads)

    def one(s, T):
        full = inputs.bench_bits(s, heads * T * D).reshape(1, heads, T, D)
        return np.ascontiguousarray(full[:, h0:h0 + hc])
    return one(seed + 2, Lq), one(seed + 3, Lk), one(seed + 4, Lk)
