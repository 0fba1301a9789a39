"""The fused attention called with host buffers: q, k, v in pinned host memory
in, the output in pinned host memory out.

A caller whose tensors live on the host (a render engine that stages its
latents in system memory, or the benchmark's end-to-end measurement) would
otherwise copy all of q, k and v to the device, run the call, and copy the
output back, one after the other.  Heads are independent, so ``HostAttention``
splits the call into head blocks (the C ABI's ``head_begin`` / ``head_count``)
and runs three streams: the host-to-device copy of block i+1, the attention of
block i (``ltxattn_fwd``) and the device-to-host copy of block i-1 overlap.
Each block is an ordinary ``ltxattn_fwd`` call over its heads, so the result is
bit-identical to the same head-block calls made on device buffers.  Against one
call over all heads it is bit-identical whenever neither splits a unit's KV
range (``num_splits=1`` guarantees that); otherwise the planner may split the
smaller block calls differently, and the two agree within the bf16 tolerance
of a split (partials combined in fp32).
"""
from __future__ import annotations

import math
from typing import List, Optional

import torch

from .backend import AttentionBackend, Failure, PreparedAttention, Rotary


def tapered_blocks(heads: int, smallest: int = 2) -> List[int]:
    """Head-block sizes that halve down to ``smallest``: 32 heads -> 16, 8, 4, 2, 2.

    Only the last block's attention and output copy run after the input copies
    end, so a small last block shortens that tail, while large early blocks keep
    the number of copies (each with a fixed cost on the copy engine) low."""
    sizes, left = [], heads
    while left > smallest:
        b = max(smallest, left // 2)
        sizes.append(b)
        left -= b
    if left > 0:
        sizes.append(left)
    return sizes


class HostAttention:
    """Device staging buffers and per-block prepared calls for one shape.

    ``q``, ``k``, ``v``: the device tensors ([B, H, T, D], contiguous) that the
    host data is copied into; ``chunks``: how many equal head blocks to
    pipeline, or ``blocks``: the head-block sizes in order (summing to H; see
    ``tapered_blocks``); ``num_splits``: passed to every block call (0 lets the
    planner choose).  Rotary tables, key mask and gate stay on the device (they
    are small and reused across calls)."""

    def __init__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: Optional[float] = None,
                 key_mask: Optional[torch.Tensor] = None, q_rotary: Optional[Rotary] = None,
                 k_rotary: Optional[Rotary] = None, chunks: int = 4, num_splits: int = 0,
                 blocks: Optional[List[int]] = None):
        for name, t in (("q", q), ("k", k), ("v", v)):
            if not t.is_cuda or not t.is_contiguous() or t.dim() != 4:
                raise Failure.shape(name, t.shape, "a contiguous CUDA [B, H, T, D]")
        B, H = q.shape[0], q.shape[1]
        if B != 1:
            raise Failure.shape("q", q.shape, "batch 1 (head blocks must be contiguous in memory)")
        if k.shape[1] != H:
            raise Failure.shape("k", k.shape, f"{H} heads (grouped KV heads are not pipelined)")
        self.q, self.k, self.v = q, k, v
        self.out = torch.empty_like(q)
        if blocks is not None:
            if any(b < 1 for b in blocks) or sum(blocks) != H:
                raise Failure.shape("blocks", tuple(blocks), f"positive head counts summing to {H}")
            starts = [sum(blocks[:i]) for i in range(len(blocks))]
            self.blocks = list(zip(starts, blocks))
        else:
            n = max(1, min(chunks, H))
            per = math.ceil(H / n)
            self.blocks = [(h, min(per, H - h)) for h in range(0, H, per)]
        self.calls: List[PreparedAttention] = [
            AttentionBackend.prepare(q, k, v, scale, key_mask=key_mask, q_rotary=q_rotary, k_rotary=k_rotary,
                                     head_begin=h0, head_count=hc, num_splits=num_splits, out=self.out)
            for h0, hc in self.blocks]
        self.h2d = torch.cuda.Stream()
        self.comp = torch.cuda.Stream()
        self.d2h = torch.cuda.Stream()

    def run(self, hq: torch.Tensor, hk: torch.Tensor, hv: torch.Tensor, hout: torch.Tensor, stream=None):
        """Copy host q, k, v in, attend, copy the output to ``hout``; ordered after and
        before the work of ``stream`` (default: the current stream)."""
        s = stream if stream is not None else torch.cuda.current_stream()
        start = torch.cuda.Event()
        start.record(s)
        for st in (self.h2d, self.comp, self.d2h):
            st.wait_event(start)
        done_in, done_attn = [], []
        for (h0, hc) in self.blocks:
            with torch.cuda.stream(self.h2d):
                for dev, host in ((self.q, hq), (self.k, hk), (self.v, hv)):
                    dev[:, h0:h0 + hc].copy_(host[:, h0:h0 + hc], non_blocking=True)
                e = torch.cuda.Event()
                e.record(self.h2d)
                done_in.append(e)
        for (h0, hc), call, e_in in zip(self.blocks, self.calls, done_in):
            self.comp.wait_event(e_in)
            call.run(self.comp)
            e = torch.cuda.Event()
            e.record(self.comp)
            done_attn.append(e)
        for (h0, hc), e_attn in zip(self.blocks, done_attn):
            self.d2h.wait_event(e_attn)
            with torch.cuda.stream(self.d2h):
                hout[:, h0:h0 + hc].copy_(self.out[:, h0:h0 + hc], non_blocking=True)
        end = torch.cuda.Event()
        end.record(self.d2h)
        s.wait_event(end)
        return hout
