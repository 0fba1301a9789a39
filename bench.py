"""Benchmark of the LTX 2.5 DiT fused attention on B200 (libltxattn_cuda).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c2|c3|c4a|c4b|c4c|c5]

Default workload (the metric's configuration): video
self-attention at the 640x384x97 render shape -- 3120 tokens, 32 heads, D=128,
bf16, q/k/v seeded N(0,1) with per-head RMSNorm, 3D split-RoPE fused into the
call, scale 1/sqrt(128), no mask.  One step = one ltxattn_fwd call.

Multi-GPU (torchrun, one process per GPU): heads are the independent units.
For c2..c4c each rank runs its own 32-head block of a (32*N)-head job (weak
scaling, no collective on the data path).  --workload c5 is the 29760-token
shape with its 32 heads sharded 32/N per rank (strong scaling).

FLOPs: 4*B*H*Lq*Lk*D per forward (the reference's convention,
Sources/ltx/BenchGEMM.swift:289).  Prints one JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "ltx-2.5-swift_b200"))

import numpy as np  # noqa: E402

WORKLOADS = {
    # name: (B, H, Lq, Lk, D, rope, mask_valid, description)
    "c2": (1, 32, 3120, 3120, 128, "3d", None, "video self-attn 640x384x97, 3120 tok, H32 D128, 3D RoPE"),
    "c3": (1, 32, 3120, 1024, 128, None, 94, "text cross-attn Q3120 x KV1024 (94 valid), H32 D128"),
    "c4a": (1, 32, 126, 126, 64, "1d", None, "audio self-attn 126 tok, H32 D64, 1D RoPE"),
    "c4b": (1, 32, 3120, 126, 64, "av", None, "video->audio cross Q3120 x KV126, H32 D64, time RoPE"),
    "c4c": (1, 32, 126, 3120, 64, "va", None, "audio->video cross Q126 x KV3120, H32 D64, time RoPE"),
    "c5": (1, 32, 29760, 29760, 128, None, None, "video self-attn 1280x768x241, 29760 tok, H32 D128"),
}
L2_BYTES = 126 * 1024 * 1024


# the roofline that bounds each workload's attention kernel (the workload's arithmetic
# intensity against the ~250 FLOP/B ridge of the measured peaks)
BOUND = {"c2": "tensor", "c3": "hbm", "c4a": "hbm", "c4b": "hbm", "c4c": "hbm", "c5": "tensor"}


# DRAM bytes per attention launch measured by ncu (profiles/fwd_bf16_sm100_c2.md)
TRAFFIC = {"c2": 83.2e6}


class L2Flush:
    """Evicts the inputs from L2 between timed steps: a write of a buffer twice
    the L2 size, then a read of a second such buffer, so a timed kernel starts
    with nothing of its own cached and with no dirty flush lines left for it to
    write back (a write-only flush leaves ~126 MB of them, which an HBM-bound
    kernel would then pay for)."""

    def __init__(self, torch):
        self.torch = torch
        self.w = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device="cuda")
        self.r = torch.ones(2 * L2_BYTES // 4, dtype=torch.float32, device="cuda")
        self.sink = torch.empty((), dtype=torch.float32, device="cuda")

    def __call__(self):
        self.w.zero_()
        self.torch.sum(self.r, dim=0, out=self.sink)


L2_NOTE = "flushed before every timed step (256 MB write, then a 256 MB read of a second buffer), outside the timed events"


def algorithmic_bytes(wl, B, H, Lq, Lk, D):
    """Bytes one attention launch must move: Q and O, plus K and V of the valid keys (bf16)."""
    valid = WORKLOADS[wl][6] or Lk
    return 2 * (2 * B * H * Lq * D + 2 * B * H * valid * D)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), d["hbm_gbs"], "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


class Clocks:
    """nvidia-smi sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for ln in f:
                parts = [x.strip() for x in ln.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = max(float(r[2]) for r in rows if r[2].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(rows)}


def make_inputs(wl, rank, Hc, B, Lq, Lk, D):
    from ltxattn import inputs
    seed = 1000 + 97 * rank
    rms = wl != "c5"  # config 5 takes config 1's inputs: plain seeded N(0,1)
    q = inputs.seeded_tensor(seed + 2, (B, Hc, Lq, D), rmsnorm=rms, bf16=True)
    k = inputs.seeded_tensor(seed + 3, (B, Hc, Lk, D), rmsnorm=rms, bf16=True)
    v = inputs.seeded_tensor(seed + 4, (B, Hc, Lk, D), bf16=True)
    rope = WORKLOADS[wl][5]
    tabs = None
    if rope == "3d":
        tabs = (inputs.rope3d_grid(13, 12, 20, D), None)
    elif rope == "1d":
        tabs = (inputs.rope1d(np.arange(Lq, dtype=np.float64), D), None)
    elif rope == "av":
        tabs = (inputs.rope1d(inputs.video_frame_seconds(13, 240), D),
                inputs.rope1d(inputs.audio_token_seconds(Lk), D))
    elif rope == "va":
        tabs = (inputs.rope1d(inputs.audio_token_seconds(Lq), D),
                inputs.rope1d(inputs.video_frame_seconds(13, 240), D))
    mask = None
    mv = WORKLOADS[wl][6]
    if mv is not None:
        mask = np.zeros((B, Lk), np.uint8)
        mask[:, :mv] = 1
    return q, k, v, tabs, mask


def run_qkprep(args):
    """q and k preparation (ltxattn_qk_prep: rmsNorm over the inner dim, head split,
    split RoPE) at the config-2 shape; GB/s against the HBM roofline."""
    import torch
    import torch.distributed as dist
    from ltxattn import Rotary, qk_prep_pair

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    if ws > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    from ltxattn import inputs
    B, H, T, D = 1, 32, 3120, 128
    inner = H * D
    seed = 1000 + 97 * rank
    xs = [torch.from_numpy(inputs.seeded_tensor(seed + i, (B, T, inner))).to("cuda", torch.bfloat16) for i in (2, 3)]
    w = torch.ones(inner, device="cuda", dtype=torch.bfloat16)
    c, sn = inputs.rope3d_grid(13, 12, 20, D)
    rot = Rotary(torch.from_numpy(c).to("cuda", torch.bfloat16), torch.from_numpy(sn).to("cuda", torch.bfloat16))
    outs = [torch.empty((B, H, T, D), device="cuda", dtype=torch.bfloat16) for _ in range(2)]
    flush = L2Flush(torch)
    stream = torch.cuda.current_stream()

    def step():  # q and k in one launch (ltxattn_qk_prep_pair)
        qk_prep_pair(xs[0], w, xs[1], w, H, rot, rot, eps=1e-6, out_q=outs[0], out_k=outs[1], stream=stream)

    def barrier():
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()

    clocks = Clocks(local)
    clocks.start()
    for _ in range(args.warmup):
        step()
    barrier()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for i in range(args.steps):
        flush()
        evs[i][0].record(stream)
        step()
        evs[i][1].record(stream)
    barrier()
    clk = clocks.stop()
    step_ms = [a.elapsed_time(b) for a, b in evs]
    # end to end: host rows in, host heads out
    hx = [x.cpu().pin_memory() for x in xs]
    ho = [torch.empty(o.shape, dtype=o.dtype).pin_memory() for o in outs]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(stream)
    for _ in range(args.steps):
        for x, h in zip(xs, hx):
            x.copy_(h, non_blocking=True)
        step()
        for o, h in zip(outs, ho):
            h.copy_(o, non_blocking=True)
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    vals = torch.tensor([sum(step_ms), e2e_ms], device="cuda", dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    total_ms, e2e_ms = vals.tolist()
    ms = total_ms / args.steps
    # algorithmic bytes per step: x in, heads out, the shared tables (cos and sin) once per tensor
    per_tensor = 2 * B * T * inner * 2 + 2 * T * (D // 2) * 2 + inner * 2
    step_bytes = 2 * per_tensor
    gbs = step_bytes * ws / (ms * 1e-3) / 1e9
    _, _, hbm, src = peaks()
    result = None
    if rank == 0:
        result = {
            "metric": "q/k prep GB/s (rmsNorm over 4096 + head split + 3D RoPE) @3120 tok (aggregate over GPUs)",
            "value": round(gbs, 1), "unit": "GB/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded N(0,1), unit norm weight, bf16)",
            "config": {"workload": "qkprep: q and k of config 2, [1, 3120, 4096] -> [1, 32, 3120, 128]",
                       "parallelism": f"heads x{ws}", "l2": L2_NOTE},
            "roofline": {"bound": "hbm", "achieved": round(gbs / ws, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(gbs / ws / hbm, 4), "peak_source": f"{src} hbm_gbs",
                         "algorithmic_bytes": step_bytes, "kernel": "qk_prep_bulk_pair_kernel", "traffic": None},
            "step_ms": {"median": round(statistics.median(step_ms), 5), "min": round(min(step_ms), 5),
                        "max": round(max(step_ms), 5)},
            "e2e": {"value": round(step_bytes * ws / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                    "h2d_bytes_per_step": sum(h.numel() * 2 for h in hx),
                    "d2h_bytes_per_step": sum(h.numel() * 2 for h in ho)},
            "gpu_launches": args.steps,
            "clocks": clk,
        }
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


def run_module(args):
    """One whole video self-attention module (DiTAttention.callAsFunction) at the
    config-2 shape: x [1, 3120, 4096] -> [1, 3120, 4096], 32 heads of 128, biases,
    q/k norms, the gate, 3D RoPE.  Projections on the library GEMM, the rest in
    libltxattn_cuda.  TFLOP/s of the module's GEMM + attention FLOPs."""
    import torch
    import torch.distributed as dist
    from ltxattn import DiTAttentionModule, Rotary, inputs

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    if ws > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    B, T, H, D = 1, 3120, 32, 128
    dim = inner = H * D
    g = torch.Generator(device="cuda").manual_seed(1000 + 97 * rank)
    dt = torch.bfloat16

    def mat(o, i):
        return (torch.randn((o, i), device="cuda", generator=g) / math.sqrt(i)).to(dt)

    def vec(n, lo=-0.1, hi=0.1):
        return (lo + (hi - lo) * torch.rand(n, device="cuda", generator=g)).to(dt)

    w = {"to_q.weight": mat(inner, dim), "to_q.bias": vec(inner), "to_k.weight": mat(inner, dim),
         "to_k.bias": vec(inner), "to_v.weight": mat(inner, dim), "to_v.bias": vec(inner),
         "to_out.0.weight": mat(dim, inner), "to_out.0.bias": vec(dim), "q_norm.weight": vec(inner, 0.5, 1.5),
         "k_norm.weight": vec(inner, 0.5, 1.5), "to_gate_logits.weight": mat(H, dim), "to_gate_logits.bias": vec(H)}
    mod = DiTAttentionModule(w, H)
    x = torch.from_numpy(inputs.seeded_tensor(1000 + 97 * rank, (B, T, dim))).to("cuda", dt)
    c, sn = inputs.rope3d_grid(13, 12, 20, D)
    rot = Rotary(torch.from_numpy(c).to("cuda", dt), torch.from_numpy(sn).to("cuda", dt))
    flush = L2Flush(torch)
    stream = torch.cuda.current_stream()
    gemm_flops = 2.0 * B * T * dim * inner * 4 + 2.0 * B * T * dim * H
    attn_flops = 4.0 * B * H * T * T * D
    flops = gemm_flops + attn_flops

    def barrier():
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()

    clocks = Clocks(local)
    clocks.start()
    for _ in range(args.warmup):
        mod(x, rotary=rot)
    barrier()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for i in range(args.steps):
        flush()
        evs[i][0].record(stream)
        mod(x, rotary=rot)
        evs[i][1].record(stream)
    barrier()
    clk = clocks.stop()
    step_ms = [a.elapsed_time(b) for a, b in evs]
    hx = x.cpu().pin_memory()
    ho = torch.empty((B, T, dim), dtype=dt).pin_memory()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(stream)
    for _ in range(args.steps):
        x.copy_(hx, non_blocking=True)
        y = mod(x, rotary=rot)
        ho.copy_(y, non_blocking=True)
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    vals = torch.tensor([statistics.median(step_ms), e2e_ms], device="cuda", dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms, e2e_ms = vals.tolist()
    burst, sustained, _, src = peaks()
    tf = flops * ws / (ms * 1e-3) / 1e12
    result = None
    if rank == 0:
        result = {
            "metric": "DiT attention module TFLOP/s bf16 (projections + fused attention) @3120-tok video self-attn "
                      "(aggregate over GPUs)",
            "value": round(tf, 1), "unit": "TFLOP/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded N(0,1) x, random-init weights of the module's shapes)",
            "config": {"workload": "module: DiTAttention attn1, x [1, 3120, 4096], 32 heads x 128, gate, 3D RoPE",
                       "parallelism": f"dp{ws}", "l2": L2_NOTE,
                       "flops_per_step": {"gemm": gemm_flops, "attention": attn_flops}},
            "roofline": {"bound": "tensor", "achieved": round(tf / ws, 1), "peak": burst, "unit": "TFLOP/s",
                         "frac": round(tf / ws / burst, 4), "peak_source": f"{src} bf16_tflops (burst)",
                         "kernel": "whole module (cuBLAS GEMMs + qk_prep + fwd_bf16_sm100_kernel)", "traffic": None},
            "e2e": {"value": round(flops * ws / (e2e_ms * 1e-3) / 1e12, 1), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": hx.numel() * 2, "d2h_bytes_per_step": ho.numel() * 2},
            "gpu_launches": 3 * args.steps,  # qk_prep for q and k, the attention (gate fused); GEMMs are cuBLAS
            "clocks": clk,
        }
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


def run_ours(args):
    import torch
    import torch.distributed as dist
    from ltxattn import AttentionBackend, Rotary, device_status

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    if ws > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    wl = args.workload
    B, H, Lq, Lk, D = WORKLOADS[wl][:5]
    strong = wl == "c5"
    if strong:
        if H % ws:
            raise SystemExit(f"{H} heads do not shard over {ws} ranks")
        Hc = H // ws
    else:
        Hc = H
    q, k, v, tabs, mask = make_inputs(wl, rank, Hc, B, Lq, Lk, D)
    dt = torch.bfloat16
    qd = torch.from_numpy(q).to("cuda", dt)
    kd = torch.from_numpy(k).to("cuda", dt)
    vd = torch.from_numpy(v).to("cuda", dt)
    out = torch.empty_like(qd)
    lse = torch.empty((B, Hc, Lq), device="cuda", dtype=torch.float32)
    qrot = krot = None
    if tabs is not None:
        qrot = Rotary(torch.from_numpy(tabs[0][0]).to("cuda", dt), torch.from_numpy(tabs[0][1]).to("cuda", dt))
        if tabs[1] is not None:
            krot = Rotary(torch.from_numpy(tabs[1][0]).to("cuda", dt), torch.from_numpy(tabs[1][1]).to("cuda", dt))
    md = torch.from_numpy(mask).cuda() if mask is not None else None
    flush = L2Flush(torch)
    stream = torch.cuda.current_stream()

    # the C-ABI call, marshalled once (AttentionBackend.prepare); each step is one ltxattn_fwd
    call = AttentionBackend.prepare(qd, kd, vd, key_mask=md, q_rotary=qrot, k_rotary=krot, out=out, lse=lse)
    kernel_call = AttentionBackend.prepare(qd, kd, vd, key_mask=md, out=out, lse=lse)

    def step():
        call.run(stream)

    # what the library launches per call (ltxattn_fwd_plan): RoPE pre-pass,
    # attention kernel, split combine
    import ctypes
    from ltxattn import _lib
    plan, kplan = _lib.FwdPlanInfo(), _lib.FwdPlanInfo()
    assert _lib.load().ltxattn_fwd_plan(ctypes.byref(call.args), ctypes.byref(plan)) == 0
    assert _lib.load().ltxattn_fwd_plan(ctypes.byref(kernel_call.args), ctypes.byref(kplan)) == 0
    launches_per_step = plan.launches
    kernel_name = "fwd_short_sm100_kernel" if kplan.kernel == 2 else "fwd_bf16_sm100_kernel"
    flops = 4.0 * B * Hc * Lq * Lk * D
    if mask is not None:
        eff_flops = 4.0 * B * Hc * Lq * WORKLOADS[wl][6] * D
    else:
        eff_flops = flops

    def barrier():
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()

    clocks = Clocks(local)
    clocks.start()
    for _ in range(args.warmup):
        step()
    barrier()
    # keep the GPU loaded for ~1.5 s so the clock sampler sees this workload under load
    t_end = time.perf_counter() + 1.5
    while time.perf_counter() < t_end:
        for _ in range(20):
            step()
        torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    for i in range(args.steps):
        flush()
        evs[i][0].record(stream)
        step()
        evs[i][1].record(stream)
    barrier()
    clk = clocks.stop()
    step_ms = [a.elapsed_time(b) for a, b in evs]
    total_ms = sum(step_ms)

    # kernel-only timing of the attention kernel: the same call without tables is one
    # launch of fwd_bf16_sm100_kernel (same shape, same FLOPs)
    kern_evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    for i in range(args.steps):
        flush()
        kern_evs[i][0].record(stream)
        kernel_call.run(stream)
        kern_evs[i][1].record(stream)
    barrier()
    kern_ms = [a.elapsed_time(b) for a, b in kern_evs]

    # end to end through the public API with host buffers
    hq = torch.from_numpy(q).to(dt).pin_memory()
    hk = torch.from_numpy(k).to(dt).pin_memory()
    hv = torch.from_numpy(v).to(dt).pin_memory()
    hout = torch.empty(out.shape, dtype=dt).pin_memory()
    e2e_steps = max(1, min(args.steps, 10))
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        qd.copy_(hq, non_blocking=True)
        kd.copy_(hk, non_blocking=True)
        vd.copy_(hv, non_blocking=True)
        step()
        hout.copy_(out, non_blocking=True)
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    h2d = (hq.numel() + hk.numel() + hv.numel()) * 2
    d2h = hout.numel() * 2
    # training backward (config 5): dQ, dK, dV from a seeded dO, P recomputed from the saved LSE
    bwd_ms = 0.0
    if args.bwd or wl == "c5":
        from ltxattn import inputs as _inp
        dout = torch.from_numpy(_inp.seeded_tensor(1000 + 97 * rank + 5, (B, Hc, Lq, D))).to("cuda", dt)
        AttentionBackend.attention(qd, kd, vd, key_mask=md, q_rotary=qrot, k_rotary=krot, out=out, lse=lse)
        grads = [torch.empty_like(qd), torch.empty_like(kd), torch.empty_like(vd)]

        def bstep():
            AttentionBackend.attention_backward(qd, kd, vd, out, dout, lse, key_mask=md, q_rotary=qrot,
                                                k_rotary=krot, dq=grads[0], dk=grads[1], dv=grads[2])
        for _ in range(args.warmup):
            bstep()
        bevs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        barrier()
        for i in range(args.steps):
            flush()
            bevs[i][0].record(stream)
            bstep()
            bevs[i][1].record(stream)
        barrier()
        bwd_ms = sum(a.elapsed_time(b) for a, b in bevs) / args.steps
    status = device_status(clear=True)

    # max over ranks
    vals = torch.tensor([total_ms, sum(kern_ms), e2e_ms, bwd_ms], device="cuda", dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    total_ms, kern_total, e2e_ms, bwd_ms = vals.tolist()
    ranks_flops = flops * ws
    ms_per_step = total_ms / args.steps
    value = ranks_flops / (ms_per_step * 1e-3) / 1e12
    kern_avg_ms = kern_total / args.steps
    burst, sustained, hbm, src = peaks()
    achieved = flops / (kern_avg_ms * 1e-3) / 1e12  # per GPU, one launch of the dominant kernel
    kern_gbs = algorithmic_bytes(wl, B, Hc, Lq, Lk, D) / (kern_avg_ms * 1e-3) / 1e9
    result = None
    if rank == 0:
        cpu = None
        if ws == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(wl, budget_s=args.cpu_seconds)
        result = {
            "metric": "fused-attn TFLOP/s bf16 @3120-tok video self-attn (aggregate over GPUs)"
            if wl == "c2" else f"fused-attn TFLOP/s bf16 ({wl})",
            "value": round(value, 2),
            "unit": "TFLOP/s",
            "n_gpus": ws,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 5),
            "higher_is_better": True,
            "scaling": "strong" if strong else "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded N(0,1), per-head RMSNorm, bf16)",
            "config": {"workload": f"{wl}: {WORKLOADS[wl][7]}", "batch": B, "heads_per_gpu": Hc,
                       "q_len": Lq, "kv_len": Lk, "head_dim": D, "rope": WORKLOADS[wl][5] or "none",
                       "mask_valid_keys": WORKLOADS[wl][6], "parallelism": f"heads x{ws}",
                       "l2": L2_NOTE,
                       "flops_per_step_per_gpu": flops, "effective_flops_per_step_per_gpu": eff_flops},
            "pct_of_datasheet_dense_bf16": round(100.0 * value / ws / 2250.0, 2),
            "value_effective_flops": round(eff_flops * ws / (ms_per_step * 1e-3) / 1e12, 3),
            "roofline": ({"bound": "tensor", "achieved": round(achieved, 2), "peak": burst, "unit": "TFLOP/s",
                          "frac": round(achieved / burst, 4), "peak_source": f"{src} bf16_tflops (burst)"}
                         if BOUND[wl] == "tensor" else
                         {"bound": "hbm", "achieved": round(kern_gbs, 1), "peak": hbm, "unit": "GB/s",
                          "frac": round(kern_gbs / hbm, 4), "peak_source": f"{src} hbm_gbs",
                          "algorithmic_bytes": algorithmic_bytes(wl, B, Hc, Lq, Lk, D),
                          "kernel_tflops": round(achieved, 2)}) | {
                         "kernel": kernel_name, "kernel_ms": round(kern_avg_ms, 5),
                         # dram__bytes_read.sum + dram__bytes_write.sum of one launch, from the ncu
                         # capture summarised in profiles/fwd_bf16_sm100_c2.md (config 2 only)
                         "traffic": TRAFFIC.get(wl)},
            "step_ms": {"median": round(statistics.median(step_ms), 5), "min": round(min(step_ms), 5),
                        "max": round(max(step_ms), 5),
                        "spread": round((max(step_ms) - min(step_ms)) / statistics.median(step_ms), 4)},
            "e2e": {"value": round(ranks_flops / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                    "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
            "device_status": status,
            "cpu_baseline": cpu,
        }
        if bwd_ms > 0:
            bflops = 2.5 * flops * ws
            result["backward"] = {"ms_per_step": round(bwd_ms, 4), "value": round(bflops / (bwd_ms * 1e-3) / 1e12, 2),
                                  "unit": "TFLOP/s", "flop_convention": "2.5 x forward (dQ, dK, dV)",
                                  "kernels": "bwd_prep_kernel, bwd_dq_kernel, bwd_dkdv_kernel"}
            result["fwd_plus_bwd_tflops"] = round(3.5 * flops * ws / ((ms_per_step + bwd_ms) * 1e-3) / 1e12, 2)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


def cpu_baseline(wl, budget_s=12.0, threads=None):
    """The oracle's fp32 explicit-path restatement on the host cores, over a
    bounded sample of heads of the same workload; TFLOP/s."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # test/baseline infrastructure; never on the GPU path
    B, H, Lq, Lk, D = WORKLOADS[wl][:5]
    threads = threads or os.cpu_count() or 1
    q, k, v, tabs, mask = make_inputs(wl, 0, 1, B, Lq, Lk, D)
    if tabs is not None:
        kt = tabs[1] if tabs[1] is not None else tabs[0]
        q = oracle.rope(q, tabs[0][0], tabs[0][1], True)
        k = oracle.rope(k, kt[0], kt[1], True)
    oracle.attn_fwd_f32(q[:, :, :64], k, v, mask=mask, threads=threads)  # warm
    t0 = time.perf_counter()
    heads = 0
    rows = min(Lq, 512) if wl == "c5" else Lq
    while True:
        oracle.attn_fwd_f32(q[:, :, :rows], k, v, mask=mask, threads=threads)
        heads += 1
        el = time.perf_counter() - t0
        if el >= budget_s or heads >= H:
            break
    flops = 4.0 * B * heads * rows * Lk * D
    return {"value": round(flops / el / 1e12, 5), "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{heads} head(s) x {rows} query rows of {wl} ({el:.1f} s), fp32 explicit path "
                      f"(oracle/ltxattn_oracle.c oracle_attn_fwd_f32, OpenMP)"}


def run_reference(args):
    ws, rank, _ = dist_env()
    if rank != 0:
        return None
    wl = args.workload
    B, H, Lq, Lk, D = WORKLOADS[wl][:5]
    threads = os.cpu_count() or 1
    per_step = max(1.0, min(4.0, 150.0 / max(1, args.steps + args.warmup)))
    for _ in range(args.warmup):
        cpu_baseline(wl, budget_s=per_step * 0.25, threads=threads)
    samples = [cpu_baseline(wl, budget_s=per_step, threads=threads) for _ in range(args.steps)]
    vals = [s["value"] for s in samples]
    value = statistics.median(vals)
    flops_step = 4.0 * B * H * Lq * Lk * D
    return {
        "impl": "reference",
        "metric": "fused-attn TFLOP/s bf16 @3120-tok video self-attn (aggregate over GPUs)"
        if wl == "c2" else f"fused-attn TFLOP/s bf16 ({wl})",
        "value": value, "unit": "TFLOP/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(flops_step / (value * 1e12) * 1e3, 3), "higher_is_better": True,
        "scaling": "strong" if wl == "c5" else "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1), per-head RMSNorm, bf16-rounded inputs)",
        "config": {"workload": f"{wl}: {WORKLOADS[wl][7]}", "batch": B, "heads": H, "q_len": Lq, "kv_len": Lk,
                   "head_dim": D},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": samples[0]["sample"] + "; MLX (the reference's CPU path) cannot run here: "
                                   "no Swift toolchain and no MLX"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def provenance():
    """What produced the line: the repository revision (when a git checkout is
    present), whether the tree was dirty, and a digest of the library loaded."""
    import hashlib
    rev = dirty = None
    try:
        rev = subprocess.run(["git", "-C", ROOT, "rev-parse", "--short", "HEAD"], capture_output=True,
                             text=True, timeout=10).stdout.strip() or None
        if rev:
            dirty = bool(subprocess.run(["git", "-C", ROOT, "status", "--porcelain", "--untracked-files=no"],
                                        capture_output=True, text=True, timeout=10).stdout.strip())
    except (OSError, subprocess.SubprocessError):
        pass
    lib = os.path.join(ROOT, "ltx-2.5-swift_b200", "libltxattn_cuda.so")
    digest = None
    if os.path.exists(lib):
        with open(lib, "rb") as f:
            digest = hashlib.sha256(f.read()).hexdigest()[:16]
    return {"revision": rev, "dirty": dirty, "library_sha256": digest}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c2", choices=sorted(WORKLOADS) + ["qkprep", "module"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--bwd", action="store_true", help="also time the training backward")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.workload == "qkprep":
        res = (run_reference(args) if args.impl == "reference" else run_qkprep(args)) \
            if args.impl != "reference" else {"impl": "reference", "unavailable": "no CPU arm for the qkprep workload"}
    elif args.workload == "module":
        res = {"impl": "reference", "unavailable": "no CPU arm for the module workload"} \
            if args.impl == "reference" else run_module(args)
    else:
        res = run_reference(args) if args.impl == "reference" else run_ours(args)
    if res is not None:
        if "unavailable" not in res:
            res["build"] = provenance()
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
