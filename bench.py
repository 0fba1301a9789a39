"""Benchmark of the LTX 2.5 DiT fused attention on B200 (libltxattn_cuda).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c2|c3|c4a|c4b|c4c|c5|a101|benchgemm|qkprep|module|outproj]
                    [--no-extras] [--no-cpu-baseline] [--bwd]

Default workload (the metric's configuration): video
self-attention at the 640x384x97 render shape -- 3120 tokens, 32 heads, D=128,
bf16, q/k/v seeded N(0,1) with per-head RMSNorm, 3D split-RoPE fused into the
call, scale 1/sqrt(128), no mask.  One step = one ltxattn_fwd call.

Multi-GPU (torchrun, one process per GPU): the 32 heads of the one job are
sharded 32/N per rank (strong scaling; heads are independent, so the
attention itself needs no collective).  Each rank builds only its own head
block of the job's inputs.  At N > 1 the line also times the NCCL all-gather
of the head blocks (ltxattn_allgather_heads), alone and after the call.

The default run adds sub-records ("extra") for the other configurations --
config 3, 4a/4b/4c, config 5 (29,760 tokens, forward and training backward)
and the config-2 backward -- each with its own roofline and a parity check of
its timed output against the CPU oracle.

FLOPs: 4*B*H*Lq*Lk*D per forward (the reference's convention,
Sources/ltx/BenchGEMM.swift:289); backward 2.5x.  Prints one JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "ltx-2.5-swift_b200"))

import numpy as np  # noqa: E402

from ltxattn.workloads import (BENCH_GEMM_CASES, DEFAULT_SEED, WORKLOADS, bench_gemm_inputs,  # noqa: E402
                               host_dout, host_inputs)

L2_BYTES = 126 * 1024 * 1024
L2_NOTE = "flushed before every timed step (256 MB write, then a 256 MB read of a second buffer), outside the timed events"
EXTRAS = ("c3", "c4a", "c4b", "c4c", "c5")

# dram__bytes_read.sum + dram__bytes_write.sum of one launch of each workload's
# attention kernel, from single-launch ncu captures of the attention call
# without tables (the kernel-only timing below), L2 flushed before the launch.
# Values for all 32 heads, from the capture summarised in the file named beside
# each number (which gives the command); scaled by heads for a rank's block.
_TRAFFIC_SRC = "ncu dram__bytes_read.sum + dram__bytes_write.sum of one L2-flushed launch (bench.py --traffic-launches)"
TRAFFIC = {"c2": (78838016, _TRAFFIC_SRC), "c3": (27749120, _TRAFFIC_SRC), "c4a": (1667840, _TRAFFIC_SRC),
           "c4b": (13884672, _TRAFFIC_SRC), "c4c": (26344704, _TRAFFIC_SRC),
           # captured on 4 of the 32 heads; scaled by heads
           "c5": (107117824 * 8, _TRAFFIC_SRC + " (4-head capture x 8)")}


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


# Launches at least this long (ms) are compared with the sustained bf16 peak.
LONG_LAUNCH_MS = 2.0


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


def metric_name(wl):
    if wl == "c2":
        return "fused-attn TFLOP/s bf16 @3120-tok video self-attn (aggregate over GPUs)"
    return f"fused-attn TFLOP/s bf16 ({wl}, aggregate over GPUs)"


def config_of(wl, ws):
    """The config block both arms print (the reference arm copies it unchanged)."""
    w = WORKLOADS[wl]
    return {"workload": f"{wl}: {w.desc}", "batch": w.B, "heads": w.H, "heads_per_gpu": w.H // ws,
            "q_len": w.Lq, "kv_len": w.Lk, "head_dim": w.D, "rope": w.rope or "none",
            "mask_valid_keys": w.mask_valid, "parallelism": f"heads x{ws}", "l2": L2_NOTE,
            "flops_per_step": w.flops, "effective_flops_per_step": w.effective_flops}


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


# ---------------------------------------------------------------------------
# the GPU arm


class Ctx:
    """Process-group, stream and flush state of one bench process."""

    def __init__(self):
        import torch
        import torch.distributed as dist
        self.torch, self.dist = torch, dist
        self.ws, self.rank, self.local = dist_env()
        torch.cuda.set_device(self.local)
        if self.ws > 1:
            from datetime import timedelta
            dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))
        self.stream = torch.cuda.current_stream()
        self.flush = L2Flush(torch)

    def barrier(self):
        if self.ws > 1:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def max_over_ranks(self, vals):
        t = self.torch.tensor(list(vals), device="cuda", dtype=self.torch.float64)
        if self.ws > 1:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return t.tolist()

    def timed(self, fn, steps, warmup=0):
        """Per-step CUDA-event times (ms) of fn on the current stream, L2 flushed before each step."""
        torch = self.torch
        for _ in range(warmup):
            fn()
        self.barrier()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for i in range(steps):
            self.flush()
            evs[i][0].record(self.stream)
            fn()
            evs[i][1].record(self.stream)
        self.barrier()
        return [a.elapsed_time(b) for a, b in evs]

    def close(self):
        if self.ws > 1:
            self.dist.barrier()
            self.dist.destroy_process_group()


def device_case(ctx, wl, h0, hc):
    """Device tensors of heads [h0, h0 + hc) of workload wl, plus the host copies the parity check reads."""
    torch = ctx.torch
    from ltxattn import Rotary
    w = WORKLOADS[wl]
    dt = torch.bfloat16
    case = {"w": w, "wl": wl, "h0": h0, "hc": hc, "qrot": None, "krot": None, "mask": None, "tabs": None,
            "mask_np": None}
    if wl == "c5":
        # 29,760 tokens x 32 heads would take minutes on the host generator: draw
        # N(0,1) on the device, one generator per head so every rank's block is
        # the same as in the single-GPU job
        def gen(off, T):
            out = torch.empty((w.B, hc, T, w.D), device="cuda", dtype=dt)
            g = torch.Generator(device="cuda")
            for i in range(hc):
                g.manual_seed(DEFAULT_SEED + 1000 * (h0 + i) + off)
                out[:, i] = torch.randn((w.B, T, w.D), device="cuda", generator=g).to(dt)
            return out
        case.update(q=gen(2, w.Lq), k=gen(3, w.Lk), v=gen(4, w.Lk), dout_fn=lambda: gen(5, w.Lq))
        case["data"] = "synthetic (N(0,1) from a seeded CUDA generator per head, bf16)"
        return case
    q, k, v, tabs, mask = host_inputs(w, heads=(h0, hc))
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dt)
    case.update(q=dev(q), k=dev(k), v=dev(v), host=(q, k, v), tabs=tabs, mask_np=mask,
                dout_fn=lambda: dev(host_dout(w, heads=(h0, hc))))
    if tabs is not None:
        case["qrot"] = Rotary(dev(tabs[0][0]), dev(tabs[0][1]))
        if tabs[1] is not None:
            case["krot"] = Rotary(dev(tabs[1][0]), dev(tabs[1][1]))
    if mask is not None:
        case["mask"] = torch.from_numpy(mask).cuda()
    case["data"] = "synthetic (seeded N(0,1) splitmix64 stream, per-head RMSNorm, bf16)"
    return case


def _oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # the checker (test infrastructure); never on the timed path
    return oracle


def parity_check(ctx, case, out, rows=512):
    """Local head 0 of the timed output against the CPU oracle (fp64 accumulation).

    Every row for the short configurations; for config 5 a sample of `rows`
    query rows (first, middle and last blocks) over all keys."""
    orc = _oracle()
    w = case["w"]
    hq = case["q"][:, :1].float().cpu().numpy()
    hk = case["k"][:, :1].float().cpu().numpy()
    hv = case["v"][:, :1].float().cpu().numpy()
    got = out[:, :1].float().cpu().numpy()
    sel = np.arange(w.Lq)
    if w.Lq > 4096:
        mid = w.Lq // 2 - rows // 4
        sel = np.concatenate([np.arange(rows // 4), np.arange(mid, mid + rows // 2), np.arange(w.Lq - rows // 4, w.Lq)])
    tabs = case["tabs"]
    q_rot = k_rot = None
    if tabs is not None:
        q_rot = (tabs[0][0][:, :, sel], tabs[0][1][:, :, sel])
        k_rot = tabs[1] if tabs[1] is not None else tabs[0]
    ref, _ = orc.attention_reference(hq[:, :, sel], hk, hv, mask=case["mask_np"], q_rot=q_rot, k_rot=k_rot,
                                     bf16=True)
    err = np.abs(got[:, :, sel].astype(np.float64) - ref)
    max_abs = float(err.max())
    rel = float(np.linalg.norm(err) / max(np.linalg.norm(ref), 1e-30))
    max_abs, rel = ctx.max_over_ranks([max_abs, rel])
    return {"max_abs": round(max_abs, 6), "rel_l2": round(rel, 6), "ok": bool(max_abs <= 2e-2 and rel <= 1e-2),
            "checked": f"head {case['h0']} of each rank, {len(sel)} of {w.Lq} query rows, fp64 oracle",
            "tolerance": "max abs 2e-2, rel-L2 1e-2"}


def bwd_parity_check(ctx, case, out, lse, grads):
    """dQ, dK, dV of local head 0 against the oracle's VJP (short configurations only)."""
    orc = _oracle()
    q, k, v = case["host"]
    do = ctx.dout_host
    q, k, v, do = q[:, :1], k[:, :1], v[:, :1], do[:, :1]
    tabs = case["tabs"]
    if tabs is not None:
        kt = tabs[1] if tabs[1] is not None else tabs[0]
        qo, ko = orc.rope(q, tabs[0][0], tabs[0][1], True), orc.rope(k, kt[0], kt[1], True)
    else:
        qo, ko = q, k
    rq, rk, rv = orc.attn_bwd(qo, ko, v, do, mask=case["mask_np"])
    if tabs is not None:
        rq, rk = orc.rope_bwd(rq, tabs[0][0], tabs[0][1], True), orc.rope_bwd(rk, kt[0], kt[1], True)
    worst_abs = worst_rel = 0.0
    for g, r in zip(grads, (rq, rk, rv)):
        e = np.abs(g[:, :1].float().cpu().numpy().astype(np.float64) - r)
        scale = max(1.0, float(np.abs(r).max()))
        worst_abs = max(worst_abs, float(e.max()) / scale)
        worst_rel = max(worst_rel, float(np.linalg.norm(e) / max(np.linalg.norm(r), 1e-3 * np.sqrt(r.size))))
    worst_abs, worst_rel = ctx.max_over_ranks([worst_abs, worst_rel])
    return {"max_abs_over_scale": round(worst_abs, 6), "rel_l2": round(worst_rel, 6),
            "ok": bool(worst_abs <= 2e-2 and worst_rel <= 1e-2),
            "checked": f"dq, dk, dv of head {case['h0']} of each rank, fp64 oracle VJP"}


def measure(ctx, args, wl, *, main=False, bwd=False):
    """Time one workload's forward (the call with its tables, and the attention
    kernel alone) on this rank's head block; optionally the backward.  Returns
    the record (rank 0) with values aggregated over ranks."""
    import ctypes
    torch = ctx.torch
    from ltxattn import AttentionBackend, _lib
    w = WORKLOADS[wl]
    if w.H % ctx.ws:
        raise SystemExit(f"{w.H} heads do not shard over {ctx.ws} ranks")
    hc = w.H // ctx.ws
    h0 = ctx.rank * hc
    case = device_case(ctx, wl, h0, hc)
    q, k, v = case["q"], case["k"], case["v"]
    out = torch.empty_like(q)
    lse = torch.empty(q.shape[:3], device="cuda", dtype=torch.float32)
    call = AttentionBackend.prepare(q, k, v, key_mask=case["mask"], q_rotary=case["qrot"], k_rotary=case["krot"],
                                    out=out, lse=lse)
    kcall = AttentionBackend.prepare(q, k, v, key_mask=case["mask"], out=out, lse=lse)
    plan, kplan = _lib.FwdPlanInfo(), _lib.FwdPlanInfo()
    assert _lib.load().ltxattn_fwd_plan(ctypes.byref(call.args), ctypes.byref(plan)) == 0
    assert _lib.load().ltxattn_fwd_plan(ctypes.byref(kcall.args), ctypes.byref(kplan)) == 0
    kernel_name = {0: "fwd_f32_kernel", 1: "fwd_bf16_sm100_kernel", 2: "fwd_short_sm100_kernel",
                   3: "fwd_persist_sm100_kernel"}[kplan.kernel]
    # Each call is captured once into a CUDA graph and replayed per step (what a
    # render or training loop that captures its DiT step does): the launches of
    # the call (RoPE pre-pass, attention, combine) then cost one graph launch.
    call.run(ctx.stream)
    kcall.run(ctx.stream)
    torch.cuda.synchronize()

    def graph_of(c):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            c.run(side)
        torch.cuda.current_stream().wait_stream(side)
        return g

    g_call, g_kern = graph_of(call), graph_of(kcall)
    run = g_call.replay
    krun = g_kern.replay

    clocks = None
    if main:
        clocks = Clocks(ctx.local)
        clocks.start()
        for _ in range(args.warmup):
            run()
        ctx.barrier()
        # keep the GPU loaded for ~1.5 s so the clock sampler sees this workload under load
        t_end = time.perf_counter() + 1.5
        while time.perf_counter() < t_end:
            for _ in range(20):
                run()
            torch.cuda.synchronize()
    step_ms = ctx.timed(run, args.steps, warmup=args.warmup)
    clk = clocks.stop() if clocks else None
    kern_ms = ctx.timed(krun, args.steps, warmup=2)
    # the timed call's output (same inputs, same tables) is what the parity check reads
    run()
    torch.cuda.synchronize()
    parity = parity_check(ctx, case, out)

    ms_rank, kern_rank = sum(step_ms) / args.steps, sum(kern_ms) / args.steps
    ms, kern = ctx.max_over_ranks([ms_rank, kern_rank])
    flops_rank = w.flops / ctx.ws
    value = w.flops / (ms * 1e-3) / 1e12
    burst, sustained, hbm, src = peaks()
    achieved_tf = flops_rank / (kern * 1e-3) / 1e12
    kern_gbs = w.algorithmic_bytes(hc) / (kern * 1e-3) / 1e9
    tr = TRAFFIC.get(wl)
    # a launch of several milliseconds runs under the 1 kW power cap for most of
    # its time, as the sustained GEMM figure does; a short launch is compared with
    # the burst figure
    long_launch = kern >= LONG_LAUNCH_MS
    tpeak, tname = (sustained, "sustained") if long_launch else (burst, "burst")
    roof = ({"bound": "tensor", "achieved": round(achieved_tf, 2), "peak": tpeak, "unit": "TFLOP/s",
             "frac": round(achieved_tf / tpeak, 4), "peak_source": f"{src} bf16_tflops ({tname})",
             "frac_of_burst": round(achieved_tf / burst, 4)}
            if w.bound == "tensor" else
            {"bound": "hbm", "achieved": round(kern_gbs, 1), "peak": hbm, "unit": "GB/s",
             "frac": round(kern_gbs / hbm, 4), "peak_source": f"{src} hbm_gbs",
             "kernel_tflops": round(achieved_tf, 2)})
    roof.update({"kernel": kernel_name, "kernel_ms": round(kern, 5),
                 "algorithmic_bytes": w.algorithmic_bytes(hc),
                 "traffic": tr[0] * hc / w.H if tr else None,
                 "traffic_source": tr[1] if tr else None})
    rec = {
        "value": round(value, 3), "unit": "TFLOP/s", "ms_per_step": round(ms, 5),
        "value_effective_flops": round(w.effective_flops / (ms * 1e-3) / 1e12, 3),
        "pct_of_datasheet_dense_bf16": round(100.0 * value / ctx.ws / 2250.0, 2),
        "roofline": roof,
        "step_ms": {"median": round(statistics.median(step_ms), 5), "min": round(min(step_ms), 5),
                    "max": round(max(step_ms), 5),
                    "spread": round((max(step_ms) - min(step_ms)) / statistics.median(step_ms), 4)},
        "launches_per_step": plan.launches, "kernel_launches_per_step": kplan.launches,
        "step_launch": "each timed step replays a CUDA graph of the call (captured once after warm-up)",
        "splits": plan.splits, "parity": parity, "data": case["data"], "config": config_of(wl, ctx.ws),
    }
    if clk is not None:
        rec["clocks"] = clk
    if bwd:
        rec["backward"] = measure_backward(ctx, args, case, out, lse)
    case["call"] = call
    return rec, case


def measure_backward(ctx, args, case, out, lse):
    torch = ctx.torch
    from ltxattn import AttentionBackend
    w = case["w"]
    q, k, v = case["q"], case["k"], case["v"]
    dout = case["dout_fn"]()
    if "host" in case:
        ctx.dout_host = dout.float().cpu().numpy()
    AttentionBackend.attention(q, k, v, key_mask=case["mask"], q_rotary=case["qrot"], k_rotary=case["krot"],
                               out=out, lse=lse)
    grads = [torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)]

    def bstep():
        AttentionBackend.attention_backward(q, k, v, out, dout, lse, key_mask=case["mask"], q_rotary=case["qrot"],
                                            k_rotary=case["krot"], dq=grads[0], dk=grads[1], dv=grads[2],
                                            stream=ctx.stream)
    bms = ctx.timed(bstep, args.steps, warmup=args.warmup)
    ms = ctx.max_over_ranks([sum(bms) / args.steps])[0]
    burst, _, _, src = peaks()
    value = 2.5 * w.flops / (ms * 1e-3) / 1e12
    rec = {"ms_per_step": round(ms, 4), "value": round(value, 2), "unit": "TFLOP/s",
           "flop_convention": "2.5 x forward (dQ, dK, dV)",
           "kernels": "bwd_prep_kernel, bwd_sm100_kernel (dK/dV and dQ passes in one launch)",
           "frac_of_burst": round(value / ctx.ws / burst, 4), "peak_source": f"{src} bf16_tflops (burst)"}
    if ms >= LONG_LAUNCH_MS:
        _, sustained, _, _ = peaks()
        rec["frac_of_sustained"] = round(value / ctx.ws / sustained, 4)
    if "host" in case:
        rec["parity"] = bwd_parity_check(ctx, case, out, lse, grads)
    return rec


def measure_e2e(ctx, args, case):
    """The same call through the public API with host buffers: q, k, v in pinned
    host memory in, the output in pinned host memory out, every copy inside the
    timed region.  ltxattn.host.HostAttention splits the call into head blocks
    and overlaps each block's host-to-device copy, attention and device-to-host
    copy on three streams (the result is bit-identical to one call)."""
    torch = ctx.torch
    from ltxattn.host import HostAttention, tapered_blocks
    q, k, v = case["q"], case["k"], case["v"]
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    hout = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    # head blocks pay off when the output copy is large enough to overlap the
    # input copies (configs 2, 3, 4b, 5); a small output (config 4a, or 4c's 126
    # query rows) leaves nothing to overlap, and more blocks only add copies and
    # launches.  The blocks taper (32 heads: 16, 8, 4, 2, 2): few copies, and a
    # small last block whose attention and output copy follow the input copies
    blocks = tapered_blocks(q.shape[1]) if hout.numel() * hout.element_size() >= (4 << 20) else [q.shape[1]]
    ha = HostAttention(q, k, v, key_mask=case["mask"], q_rotary=case["qrot"], k_rotary=case["krot"], blocks=blocks)
    ha.run(hq, hk, hv, hout, stream=ctx.stream)  # warm
    steps = max(1, min(args.steps, 10))
    ctx.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(ctx.stream)
    for _ in range(steps):
        ha.run(hq, hk, hv, hout, stream=ctx.stream)
    e1.record(ctx.stream)
    ctx.barrier()
    ms = ctx.max_over_ranks([e0.elapsed_time(e1) / steps])[0]
    # the host output against the device call's output (same inputs and tables):
    # the head-block calls may split KV ranges differently from one call, so the
    # two agree within the bf16 tolerance of a split, not bit for bit
    torch.cuda.synchronize()
    ref = case["call"].out.float().cpu()
    err = (hout.float() - ref).abs()
    max_abs = float(err.max())
    rel = float(err.norm() / max(float(ref.norm()), 1e-30))
    max_abs, rel = ctx.max_over_ranks([max_abs, rel])
    w = case["w"]
    return {"value": round(w.flops / (ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s", "ms_per_step": round(ms, 4),
            "check": {"against": "the device call's output", "max_abs": round(max_abs, 6), "rel_l2": round(rel, 6),
                      "ok": bool(max_abs <= 2e-2 and rel <= 1e-2)},
            "h2d_bytes_per_step": (hq.numel() + hk.numel() + hv.numel()) * 2,
            "d2h_bytes_per_step": hout.numel() * 2,
            "pipeline": (f"head blocks of {','.join(map(str, blocks))} heads, H2D / attention / D2H overlapped on "
                         "three streams" if len(blocks) > 1
                         else "one block: H2D, attention, D2H on three streams in sequence")}


def measure_gather(ctx, args, case):
    """N > 1: the NCCL all-gather of the ranks' head blocks (ltxattn_allgather_heads),
    alone and right after the call ("with gather")."""
    torch = ctx.torch
    from ltxattn import dist as ldist
    uid = ldist.exchange_unique_id()
    hg = ldist.HeadGather(ctx.ws, ctx.rank, uid, ctx.local)
    try:
        nranks, nrank = hg.size()
        out = case["call"].out
        full = torch.empty((out.shape[0], out.shape[1] * ctx.ws) + tuple(out.shape[2:]), dtype=out.dtype,
                           device="cuda")
        g_ms = ctx.timed(lambda: hg.gather(out, full, stream=ctx.stream), args.steps, warmup=args.warmup)

        def both():
            case["call"].run(ctx.stream)
            hg.gather(out, full, stream=ctx.stream)
        b_ms = ctx.timed(both, args.steps, warmup=args.warmup)
        ctx.torch.cuda.synchronize()
        g, b = ctx.max_over_ranks([sum(g_ms) / args.steps, sum(b_ms) / args.steps])
    finally:
        ctx.barrier()
        hg.close()
    w = case["w"]
    total = full.numel() * full.element_size()
    fused = measure_fused_gather(ctx, args, case, full) if args.fused_gather else None
    return {"gather_ms": round(g, 5), "bytes_gathered_per_rank": total, "fused": fused,
            "algbw_gbs": round(total / (g * 1e-3) / 1e9, 1),
            "value_with_gather": round(w.flops / (b * 1e-3) / 1e12, 3), "ms_per_step_with_gather": round(b, 5),
            "nccl_nranks": nranks, "nccl_rank": nrank, "nccl_nranks_ok": nranks == ctx.ws}


def measure_fused_gather(ctx, args, case, gathered):
    """N > 1, --fused-gather: ltxattn_fwd_gather (the attention's epilogue stores
    every output tile into every rank's output over NVLink) on the same job, timed
    like "with gather", and its output checked against the call + NCCL gather."""
    torch = ctx.torch
    from ltxattn.dist import FusedHeadGather
    wl = case["wl"]
    w = case["w"]
    full_case = device_case(ctx, wl, 0, w.H)  # every head's inputs; each rank reads its block
    fg = FusedHeadGather(tuple(full_case["q"].shape))
    try:
        def run():
            fg.run(full_case["q"], full_case["k"], full_case["v"], q_rotary=full_case["qrot"],
                   k_rotary=full_case["krot"], stream=ctx.stream)
        f_ms = ctx.timed(run, args.steps, warmup=args.warmup)
        torch.cuda.synchronize()
        err = (fg.out.float() - gathered.float()).abs()
        max_abs = float(err.max())
        f, max_abs = ctx.max_over_ranks([sum(f_ms) / args.steps, max_abs])
    finally:
        fg.close()
    return {"ms_per_step": round(f, 5), "value": round(w.flops / (f * 1e-3) / 1e12, 3),
            "max_abs_vs_nccl_gather": round(max_abs, 6),
            "how": "ltxattn_fwd_gather: TMA stores of every output tile into the other ranks' outputs in the "
                   "epilogue (split rows from the combine), bounded entry and completion handshakes"}


def run_ours(args):
    from ltxattn import device_status
    ctx = Ctx()
    wl = args.workload
    rec, case = measure(ctx, args, wl, main=True, bwd=args.bwd or wl == "c5")
    e2e = measure_e2e(ctx, args, case)
    gather = measure_gather(ctx, args, case) if ctx.ws > 1 else None
    extras = {}
    if not args.no_extras and wl == "c2":
        r2b = measure_backward(ctx, args, case, case["call"].out, case["call"].lse)
        extras["c2_backward"] = r2b
        del case
        for x in EXTRAS:
            r, c = measure(ctx, args, x, bwd=(x == "c5"))
            extras[x] = r
            del c
            ctx.torch.cuda.empty_cache()
    status = device_status(clear=True)
    st = ctx.max_over_ranks([float(status)])[0]
    result = None
    if ctx.rank == 0:
        cpu = None
        if ctx.ws == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(wl, budget_s=args.cpu_seconds)
        w = WORKLOADS[wl]
        result = {
            "metric": metric_name(wl),
            "value": round(rec["value"], 2), "unit": "TFLOP/s", "n_gpus": ctx.ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": rec["ms_per_step"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": rec["data"],
            "config": rec["config"],
            "pct_of_datasheet_dense_bf16": rec["pct_of_datasheet_dense_bf16"],
            "value_effective_flops": rec["value_effective_flops"],
            "roofline": rec["roofline"], "step_ms": rec["step_ms"], "parity": rec["parity"],
            "e2e": e2e,
            "gpu_launches": rec["launches_per_step"] * args.steps,
            "clocks": rec.get("clocks"),
            "device_status": int(st),
            "cpu_baseline": cpu,
        }
        if "backward" in rec:
            result["backward"] = rec["backward"]
            result["fwd_plus_bwd_tflops"] = round(3.5 * w.flops / ((rec["ms_per_step"] + rec["backward"]["ms_per_step"])
                                                                    * 1e-3) / 1e12, 2)
        if gather is not None:
            result["gather"] = gather
        if extras:
            result["extra"] = extras
    ctx.close()
    return result


def run_benchgemm(args):
    """The reference bench's attention case set (BenchGEMM.swift:466-497) with its
    own operands (BenchOperand.bits, seed 0x5EED + 2/3/4): SDPA alone, no mask, no
    RoPE.  One line; value = the attn1.video_self case."""
    import torch
    from ltxattn import AttentionBackend
    ctx = Ctx()
    cases = []
    for name, Lq, Lk, D in BENCH_GEMM_CASES:
        hc = 32 // ctx.ws
        h0 = ctx.rank * hc
        q, k, v = (torch.from_numpy(x).to("cuda", torch.bfloat16)
                   for x in bench_gemm_inputs(Lq, Lk, D, head_range=(h0, hc)))
        call = AttentionBackend.prepare(q, k, v)
        ms = ctx.timed(lambda: call.run(ctx.stream), args.steps, warmup=args.warmup)
        med = statistics.median(ms)
        med, mn, mx = ctx.max_over_ranks([med, min(ms), max(ms)])
        flops = 4.0 * 32 * Lq * Lk * D
        cases.append({"name": name, "heads": 32, "queryTokens": Lq, "keyTokens": Lk, "headDim": D,
                      "flops": flops, "median_ms": round(med, 5), "min_ms": round(mn, 5), "max_ms": round(mx, 5),
                      "spread": round((mx - mn) / med, 4), "tflopsFromMedian": round(flops / (med * 1e-3) / 1e12, 2),
                      "tflopsFromMin": round(flops / (mn * 1e-3) / 1e12, 2)})
    result = None
    if ctx.rank == 0:
        c0 = cases[0]
        result = {"metric": "fused-attn TFLOP/s bf16, the reference bench's attention cases (attn1.video_self)",
                  "value": c0["tflopsFromMedian"], "unit": "TFLOP/s", "n_gpus": ctx.ws, "steps": args.steps,
                  "warmup": args.warmup, "ms_per_step": c0["median_ms"], "higher_is_better": True,
                  "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                  "data": "the reference bench's operands (BenchOperand.bits, seed 0x5EED)",
                  "config": {"workload": "benchgemm: BenchGEMM.swift:466-497 attention cases at 3120 video / "
                                         "101 audio / 1024 text tokens", "parallelism": f"heads x{ctx.ws}",
                             "l2": L2_NOTE},
                  "cases": cases}
    ctx.close()
    return result


# ---------------------------------------------------------------------------
# q/k preparation and the whole module (single-purpose workloads)


def run_qkprep(args):
    """q and k preparation (ltxattn_qk_prep: rmsNorm over the inner dim, head split,
    split RoPE) at the config-2 shape; GB/s against the HBM roofline."""
    import torch
    from ltxattn import Rotary, inputs, qk_prep_pair
    ctx = Ctx()
    B, H, T, D = 1, 32, 3120, 128
    inner = H * D
    seed = DEFAULT_SEED + 97 * ctx.rank
    xs = [torch.from_numpy(inputs.seeded_tensor(seed + i, (B, T, inner))).to("cuda", torch.bfloat16) for i in (2, 3)]
    w = torch.ones(inner, device="cuda", dtype=torch.bfloat16)
    c, sn = inputs.rope3d_grid(13, 12, 20, D)
    rot = Rotary(torch.from_numpy(c).to("cuda", torch.bfloat16), torch.from_numpy(sn).to("cuda", torch.bfloat16))
    outs = [torch.empty((B, H, T, D), device="cuda", dtype=torch.bfloat16) for _ in range(2)]

    def call(stream):  # q and k in one launch (ltxattn_qk_prep_pair)
        qk_prep_pair(xs[0], w, xs[1], w, H, rot, rot, eps=1e-6, out_q=outs[0], out_k=outs[1], stream=stream)

    # captured once and replayed per step, as the attention workloads are, so the
    # wrapper's host work between the start event and the launch is not timed
    call(ctx.stream)
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        call(side)
    torch.cuda.current_stream().wait_stream(side)
    step = graph.replay

    clocks = Clocks(ctx.local)
    clocks.start()
    # keep the GPU loaded for ~0.5 s first: the sampler process starts meanwhile,
    # so its start-up does not land inside a timed step
    t_end = time.perf_counter() + 0.5
    while time.perf_counter() < t_end:
        for _ in range(20):
            step()
        torch.cuda.synchronize()
    step_ms = ctx.timed(step, args.steps, warmup=args.warmup)
    clk = clocks.stop()
    hx = [x.cpu().pin_memory() for x in xs]
    ho = [torch.empty(o.shape, dtype=o.dtype).pin_memory() for o in outs]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx.barrier()
    e0.record(ctx.stream)
    for _ in range(args.steps):
        for x, h in zip(xs, hx):
            x.copy_(h, non_blocking=True)
        step()
        for o, h in zip(outs, ho):
            h.copy_(o, non_blocking=True)
    e1.record(ctx.stream)
    ctx.barrier()
    ms, e2e_ms = ctx.max_over_ranks([sum(step_ms) / args.steps, e0.elapsed_time(e1) / args.steps])
    # algorithmic bytes per step: x in, heads out, the shared tables (cos and sin) once per tensor
    per_tensor = 2 * B * T * inner * 2 + 2 * T * (D // 2) * 2 + inner * 2
    step_bytes = 2 * per_tensor
    gbs = step_bytes * ctx.ws / (ms * 1e-3) / 1e9
    _, _, hbm, src = peaks()
    result = None
    if ctx.rank == 0:
        result = {
            "metric": "q/k prep GB/s (rmsNorm over 4096 + head split + 3D RoPE) @3120 tok (aggregate over GPUs)",
            "value": round(gbs, 1), "unit": "GB/s", "n_gpus": ctx.ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded N(0,1), unit norm weight, bf16)",
            "config": {"workload": "qkprep: q and k of config 2, [1, 3120, 4096] -> [1, 32, 3120, 128]",
                       "parallelism": f"heads x{ctx.ws}", "l2": L2_NOTE},
            "roofline": {"bound": "hbm", "achieved": round(gbs / ctx.ws, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(gbs / ctx.ws / hbm, 4), "peak_source": f"{src} hbm_gbs",
                         "algorithmic_bytes": step_bytes, "kernel": "qk_prep_bulk_pair_kernel", "traffic": None},
            "step_ms": {"median": round(statistics.median(step_ms), 5), "min": round(min(step_ms), 5),
                        "max": round(max(step_ms), 5)},
            "e2e": {"value": round(step_bytes * ctx.ws / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                    "h2d_bytes_per_step": sum(h.numel() * 2 for h in hx),
                    "d2h_bytes_per_step": sum(h.numel() * 2 for h in ho)},
            "gpu_launches": args.steps,
            "clocks": clk,
        }
    ctx.close()
    return result


def run_module(args):
    """One whole video self-attention module (DiTAttention.callAsFunction) at the
    config-2 shape: x [1, 3120, 4096] -> [1, 3120, 4096], 32 heads of 128, biases,
    q/k norms, the gate, 3D RoPE.  Every launch is libltxattn_cuda's: the five
    projections on its tcgen05 GEMM (ltxattn_linear; the narrow gate logits split
    K and add a second, bias-and-round launch), qk_prep_pair, the attention.  TFLOP/s of the module's GEMM + attention FLOPs."""
    import math
    import torch
    from ltxattn import DiTAttentionModule, Rotary, inputs
    ctx = Ctx()
    B, T, H, D = 1, 3120, 32, 128
    dim = inner = H * D
    g = torch.Generator(device="cuda").manual_seed(DEFAULT_SEED + 97 * ctx.rank)
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
    x = torch.from_numpy(inputs.seeded_tensor(DEFAULT_SEED + 97 * ctx.rank, (B, T, dim))).to("cuda", dt)
    c, sn = inputs.rope3d_grid(13, 12, 20, D)
    rot = Rotary(torch.from_numpy(c).to("cuda", dt), torch.from_numpy(sn).to("cuda", dt))
    gemm_flops = 2.0 * B * T * dim * inner * 4 + 2.0 * B * T * dim * H
    attn_flops = 4.0 * B * H * T * T * D
    flops = gemm_flops + attn_flops
    clocks = Clocks(ctx.local)
    clocks.start()
    t_end = time.perf_counter() + 0.5  # the sampler starts while the GPU is loaded, not inside a timed step
    while time.perf_counter() < t_end:
        mod(x, rotary=rot)
        torch.cuda.synchronize()
    step_ms = ctx.timed(lambda: mod(x, rotary=rot), args.steps, warmup=args.warmup)
    clk = clocks.stop()
    hx = x.cpu().pin_memory()
    ho = torch.empty((B, T, dim), dtype=dt).pin_memory()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx.barrier()
    e0.record(ctx.stream)
    for _ in range(args.steps):
        x.copy_(hx, non_blocking=True)
        y = mod(x, rotary=rot)
        ho.copy_(y, non_blocking=True)
    e1.record(ctx.stream)
    ctx.barrier()
    ms, e2e_ms = ctx.max_over_ranks([statistics.median(step_ms), e0.elapsed_time(e1) / args.steps])
    burst, _, _, src = peaks()
    tf = flops * ctx.ws / (ms * 1e-3) / 1e12
    result = None
    if ctx.rank == 0:
        result = {
            "metric": "DiT attention module TFLOP/s bf16 (projections + fused attention) @3120-tok video self-attn "
                      "(aggregate over GPUs)",
            "value": round(tf, 1), "unit": "TFLOP/s", "n_gpus": ctx.ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded N(0,1) x, random-init weights of the module's shapes)",
            "config": {"workload": "module: DiTAttention attn1, x [1, 3120, 4096], 32 heads x 128, gate, 3D RoPE",
                       "parallelism": f"dp{ctx.ws}", "l2": L2_NOTE,
                       "flops_per_step": {"gemm": gemm_flops, "attention": attn_flops}},
            "roofline": {"bound": "tensor", "achieved": round(tf / ctx.ws, 1), "peak": burst, "unit": "TFLOP/s",
                         "frac": round(tf / ctx.ws / burst, 4), "peak_source": f"{src} bf16_tflops (burst)",
                         "kernel": "whole module (linear_kernel x5 + bias_round + qk_prep_pair + fwd_persist_sm100_kernel)", "traffic": None},
            "e2e": {"value": round(flops * ctx.ws / (e2e_ms * 1e-3) / 1e12, 1), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": hx.numel() * 2, "d2h_bytes_per_step": ho.numel() * 2},
            "gpu_launches": 8 * args.steps,  # v, gate (split K: 2), q, k, qk_prep_pair, attention, to_out
            "clocks": clk,
        }
    ctx.close()
    return result


def run_outproj(args):
    """Row-parallel to_out of a head-sharded module at the config-2 shape: rank r
    holds heads [r*32/N, (r+1)*32/N) of the merged attention output [3120, 4096]
    and the matching column block of to_out.0.weight [4096, 4096];
    ltxattn_out_project_allreduce (tcgen05 GEMM to an fp32 partial, NCCL
    all-reduce, bias and rounding) leaves the whole output on every rank.
    TFLOP/s of the whole to_out (2 M N K) per step; the GEMM alone and the
    all-reduce's share are reported beside it, and rank 0 checks sampled rows
    against the oracle."""
    import ctypes
    import torch
    from ltxattn import _lib
    from ltxattn import dist as ldist
    from ltxattn.proj import linear
    ctx = Ctx()
    M, N, H, D = 3120, 4096, 32, 128
    K = H * D
    if H % ctx.ws:
        raise SystemExit(f"{H} heads do not shard over {ctx.ws} ranks")
    k = (H // ctx.ws) * D
    k0 = ctx.rank * k
    g = torch.Generator(device="cuda").manual_seed(DEFAULT_SEED)  # the same tensors on every rank
    bf = torch.bfloat16
    merged = torch.randn((M, K), generator=g, device="cuda").to(bf)
    W = (torch.randn((N, K), generator=g, device="cuda") / 64).to(bf)
    b = (torch.randn(N, generator=g, device="cuda") * 0.1).to(bf)
    x_local, w_block = merged[:, k0:k0 + k], W[:, k0:k0 + k]
    if ctx.ws > 1:
        uid = ldist.exchange_unique_id()
    else:
        raw = (ctypes.c_uint8 * 128)()
        assert _lib.load().ltxattn_comm_unique_id(raw) == _lib.OK
        uid = bytes(raw)
    hg = ldist.HeadGather(ctx.ws, ctx.rank, uid, ctx.local)
    out = torch.empty((M, N), device="cuda", dtype=bf)
    wsb = torch.empty(M * N * 4, device="cuda", dtype=torch.uint8)
    try:
        nranks, _ = hg.size()
        step = lambda: hg.out_project(x_local, w_block, b, out=out, workspace=wsb, stream=ctx.stream)
        full_ms = ctx.timed(step, args.steps, warmup=args.warmup)
        part = torch.empty((M, N), device="cuda", dtype=bf)
        gemm_ms = ctx.timed(lambda: linear(x_local, w_block, out=part, stream=ctx.stream), args.steps,
                            warmup=args.warmup)
        step()
        torch.cuda.synchronize()
        parity = None
        if ctx.rank == 0:
            orc = _oracle()
            rows = np.r_[0:32, 1544:1576, 3088:3120]
            ref = orc.linear(merged[torch.as_tensor(rows, device="cuda")].float().cpu().numpy(),
                             W.float().cpu().numpy(), b.float().cpu().numpy())
            got = out[torch.as_tensor(rows, device="cuda")].float().cpu().numpy()
            err = np.abs(got - ref)
            rel = float(np.linalg.norm(err) / np.linalg.norm(ref))
            parity = {"max_abs": round(float(err.max()), 6), "rel_l2": round(rel, 6),
                      "ok": bool(err.max() <= 2e-2 and rel <= 1e-2),
                      "checked": f"{len(rows)} rows of the reduced output on rank 0, fp64 oracle of the full to_out"}
        ms, gms = ctx.max_over_ranks([sum(full_ms) / args.steps, sum(gemm_ms) / args.steps])
        fused = None
        if args.fused_gather and ctx.ws > 1:
            # ltxattn_out_project_fused: the reduction over peer memory instead of NCCL
            fo = ldist.FusedOutProject(M, N)
            try:
                f_ms = ctx.timed(lambda: fo.run(x_local, w_block, b, stream=ctx.stream), args.steps,
                                 warmup=args.warmup)
                torch.cuda.synchronize()
                same = float((fo.out.float() - out.float()).abs().max())
                fms, same = ctx.max_over_ranks([sum(f_ms) / args.steps, same])
            finally:
                fo.close()
            fused = {"ms_per_step": round(fms, 5), "value": round(2.0 * M * N * K / (fms * 1e-3) / 1e12, 2),
                     "max_abs_vs_nccl_path": round(same, 6),
                     "how": "ltxattn_out_project_fused: fp32 partial rows stored into their owners' planes by the "
                            "GEMM epilogue, owners reduce in rank order and store into every output, bounded "
                            "handshakes"}
    finally:
        ctx.barrier()
        hg.close()
    flops = 2.0 * M * N * K
    burst, _, _, src = peaks()
    result = None
    if ctx.rank == 0:
        result = {
            "metric": "row-parallel to_out TFLOP/s bf16 (tcgen05 GEMM + NCCL all-reduce) @3120 tok, 4096 -> 4096 "
                      "(aggregate over GPUs)",
            "value": round(flops / (ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s", "n_gpus": ctx.ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (N(0,1) merged output, N(0,1)/64 weight, seeded CUDA generator)",
            "config": {"workload": "outproj: to_out.0 over head shards, [3120, 4096] x [4096, 4096]^T + b",
                       "parallelism": f"heads x{ctx.ws}", "l2": L2_NOTE, "k_per_rank": k},
            "gemm_ms": round(gms, 5),
            "gemm_tflops_per_gpu": round(2.0 * M * N * k / (gms * 1e-3) / 1e12, 2),
            "gemm_frac_of_burst": round(2.0 * M * N * k / (gms * 1e-3) / 1e12 / burst, 4),
            "allreduce_and_round_ms": round(max(0.0, ms - gms), 5),
            "allreduce_bytes_per_rank": M * N * 4, "nccl_nranks": nranks,
            "parity": parity, "gpu_launches": 2 * args.steps, "fused": fused,
        }
    ctx.close()
    return result


# ---------------------------------------------------------------------------
# the CPU arms


def cpu_step(wl, q, k, v, tabs, mask, threads, rows=None):
    """One pass of the reference's explicit path on the host (oracle/ltxattn_oracle.c,
    fp32): the split RoPE of q and k, then softmax(q k^T scale) v, for the given heads."""
    orc = _oracle()
    if rows is not None:
        q = q[:, :, :rows]
    if tabs is not None:
        kt = tabs[1] if tabs[1] is not None else tabs[0]
        qt = (tabs[0][0][:, :, :q.shape[2]], tabs[0][1][:, :, :q.shape[2]])
        q = orc.rope(q, qt[0], qt[1], True)
        k = orc.rope(k, kt[0], kt[1], True)
    orc.attn_fwd_f32(q, k, v, mask=mask, threads=threads)


def cpu_baseline(wl, budget_s=12.0, threads=None):
    """The oracle's fp32 explicit-path restatement (RoPE included) on the host
    cores, over a bounded sample of heads of the same workload; TFLOP/s."""
    w = WORKLOADS[wl]
    threads = threads or os.cpu_count() or 1
    rows = min(w.Lq, 512) if wl == "c5" else None
    if wl == "c5":
        q, k, v, tabs, mask = host_inputs(w, heads=(0, 1))
    else:
        q, k, v, tabs, mask = host_inputs(w)
    cpu_step(wl, q[:, :1], k[:, :1], v[:, :1], tabs, mask, threads, rows=64)  # warm
    t0 = time.perf_counter()
    heads = 0
    while True:
        cpu_step(wl, q[:, heads:heads + 1], k[:, heads:heads + 1], v[:, heads:heads + 1], tabs, mask, threads,
                 rows=rows)
        heads += 1
        el = time.perf_counter() - t0
        if el >= budget_s or heads >= q.shape[1]:
            break
    r = rows or w.Lq
    flops = 4.0 * w.B * heads * r * w.Lk * w.D
    return {"value": round(flops / el / 1e12, 5), "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{heads} head(s) x {r} query rows of {wl} ({el:.1f} s), split RoPE + fp32 explicit path "
                      f"(oracle/ltxattn_oracle.c oracle_rope + oracle_attn_fwd_f32, OpenMP)"}


def run_reference(args):
    """The reference's CPU path for this workload, restated (MLX on CPU cannot run
    here: no Swift toolchain, no MLX): RoPE + fp32 explicit attention on all host
    cores.  Each step is the whole workload where that takes about a second or two
    (configs 2-4); config 5's step is one head x 512 query rows."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return None
    wl = args.workload
    w = WORKLOADS[wl]
    threads = os.cpu_count() or 1
    if wl == "c5":
        q, k, v, tabs, mask = host_inputs(w, heads=(0, 1))
        rows, sample = 512, "1 head x 512 query rows of 29760 per step"
        flops = 4.0 * w.B * 1 * rows * w.Lk * w.D
    else:
        q, k, v, tabs, mask = host_inputs(w)
        rows, sample = None, f"the whole workload ({w.H} heads) per step"
        flops = w.flops

    def step():
        cpu_step(wl, q, k, v, tabs, mask, threads, rows=rows)
    for _ in range(args.warmup):
        step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    value = round(flops / med / 1e12, 6)
    return {
        "impl": "reference", "metric": metric_name(wl), "value": value, "unit": "TFLOP/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(med * 1e3, 3),
        "step_ms": {"median": round(med * 1e3, 3), "min": round(min(times) * 1e3, 3),
                    "max": round(max(times) * 1e3, 3)},
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) splitmix64 stream, per-head RMSNorm, bf16-rounded inputs)",
        "config": config_of(wl, ws),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": sample + "; split RoPE + fp32 explicit path timed together "
                                   "(oracle/ltxattn_oracle.c, OpenMP); MLX (the reference's CPU path) cannot run "
                                   "here: no Swift toolchain and no MLX"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def run_traffic_launches(args):
    """One L2-flushed launch of each workload's attention call without tables
    (the kernel-only call the roofline times), in the order c2, c3, c4a, c4b,
    c4c, c5 (heads 0..3: one rank's block at 8 GPUs), for a single-pass ncu
    capture of dram__bytes per launch.  Prints the order it launched."""
    import torch
    from ltxattn import AttentionBackend
    ctx = Ctx()
    order = []
    for wl in ("c2", "c3", "c4a", "c4b", "c4c", "c5"):
        w = WORKLOADS[wl]
        hc = 4 if wl == "c5" else w.H
        case = device_case(ctx, wl, 0, hc)
        call = AttentionBackend.prepare(case["q"], case["k"], case["v"], key_mask=case["mask"], save_lse=True)
        call.run(ctx.stream)  # untraced by the capture's kernel filter order: warm the module
        torch.cuda.synchronize()
        ctx.flush()
        call.run(ctx.stream)
        torch.cuda.synchronize()
        order.append({"workload": wl, "heads": hc, "algorithmic_bytes": w.algorithmic_bytes(hc)})
        del case, call
    ctx.close()
    return {"traffic_launch_order": order, "note": "each workload launches its call twice; the second follows an L2 flush"}


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
    ap.add_argument("--workload", default="c2",
                    choices=sorted(WORKLOADS) + ["benchgemm", "qkprep", "module", "outproj"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="only the chosen workload (no sub-records)")
    ap.add_argument("--fused-gather", action="store_true",
                    help="N > 1: also time ltxattn_fwd_gather (the all-gather fused into the attention) and, "
                         "with --workload outproj, ltxattn_out_project_fused")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--bwd", action="store_true", help="also time the training backward")
    ap.add_argument("--traffic-launches", action="store_true",
                    help="one flushed launch per workload for an ncu dram__bytes capture (no timing)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.traffic_launches:
        print(json.dumps(run_traffic_launches(args)), flush=True)
        return
    if args.impl == "reference":
        if args.workload in WORKLOADS:
            res = run_reference(args)
        else:
            res = {"impl": "reference", "unavailable": f"no CPU arm for the {args.workload} workload"}
    elif args.workload == "qkprep":
        res = run_qkprep(args)
    elif args.workload == "module":
        res = run_module(args)
    elif args.workload == "benchgemm":
        res = run_benchgemm(args)
    elif args.workload == "outproj":
        res = run_outproj(args)
    else:
        res = run_ours(args)
    if res is not None:
        if "unavailable" not in res:
            res["build"] = provenance()
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
