"""The C ABI without a GPU: the library loads, exports exactly what
include/ltxattn.h declares, its structs have the layout the ctypes binding
assumes, and argument validation refuses bad calls before touching a device."""
import ctypes
import os
import re
import subprocess

import pytest

from ltxattn import _lib, backend

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "ltxattn.h")


def declared_entry_points():
    names = set()
    for h in os.listdir(os.path.join(ROOT, "include")):
        if h.endswith(".h"):
            text = open(os.path.join(ROOT, "include", h)).read()
            names |= set(re.findall(r"LTXATTN_API[^;(]*?\b(ltxattn_\w+)\s*\(", text))
    return names


def test_library_loads_and_exports_every_declared_symbol():
    L = _lib.load()
    declared = declared_entry_points()
    assert declared, "no entry points parsed from include/"
    assert set(_lib.EXPORTED) <= declared
    for name in sorted(declared):
        assert hasattr(L, name), f"{name} declared in include/ but not exported"
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln and "ltxattn_" in ln}
    assert exported == declared, f"exports differ from the header: {exported ^ declared}"
    assert L.ltxattn_abi_version() == 3


PROBE = r"""
#include <stddef.h>
#include <stdio.h>
#include "ltxattn.h"
#define P(T, f) printf(#T "." #f " %zu\n", offsetof(T, f));
int main(void) {
  printf("ltxattn_tensor %zu\n", sizeof(ltxattn_tensor));
  printf("ltxattn_rotary %zu\n", sizeof(ltxattn_rotary));
  printf("ltxattn_fwd_args %zu\n", sizeof(ltxattn_fwd_args));
  printf("ltxattn_bwd_args %zu\n", sizeof(ltxattn_bwd_args));
  printf("ltxattn_gather_args %zu\n", sizeof(ltxattn_gather_args));
  printf("ltxattn_device_info %zu\n", sizeof(ltxattn_device_info));
  printf("ltxattn_rope_args %zu\n", sizeof(ltxattn_rope_args));
  printf("ltxattn_rotary_table_args %zu\n", sizeof(ltxattn_rotary_table_args));
  printf("ltxattn_qk_prep_args %zu\n", sizeof(ltxattn_qk_prep_args));
  printf("ltxattn_fwd_plan_info %zu\n", sizeof(ltxattn_fwd_plan_info));
  printf("ltxattn_memory_plan_args %zu\n", sizeof(ltxattn_memory_plan_args));
  printf("ltxattn_linear_args %zu\n", sizeof(ltxattn_linear_args));
  printf("ltxattn_out_project_args %zu\n", sizeof(ltxattn_out_project_args));
  printf("ltxattn_head_gate_args %zu\n", sizeof(ltxattn_head_gate_args));
  printf("ltxattn_gather_peers %zu\n", sizeof(ltxattn_gather_peers));
  P(ltxattn_gather_peers, out) P(ltxattn_gather_peers, signals) P(ltxattn_gather_peers, epoch)
  printf("ltxattn_reduce_peers %zu\n", sizeof(ltxattn_reduce_peers));
  P(ltxattn_reduce_peers, recv) P(ltxattn_reduce_peers, out) P(ltxattn_reduce_peers, signals)
  P(ltxattn_reduce_peers, epoch)
  P(ltxattn_linear_args, out_stride) P(ltxattn_linear_args, workspace_bytes)
  P(ltxattn_out_project_args, workspace_bytes) P(ltxattn_head_gate_args, gate_stride_h)
  printf("ltxattn_memory_plan_info %zu\n", sizeof(ltxattn_memory_plan_info));
  P(ltxattn_memory_plan_args, resident_bytes) P(ltxattn_memory_plan_args, margin_fraction)
  P(ltxattn_memory_plan_info, fits) P(ltxattn_memory_plan_info, bytes_per_token)
  P(ltxattn_fwd_args, q) P(ltxattn_fwd_args, out) P(ltxattn_fwd_args, scale)
  P(ltxattn_fwd_args, key_mask) P(ltxattn_fwd_args, q_rotary) P(ltxattn_fwd_args, k_rotary)
  P(ltxattn_fwd_args, lse) P(ltxattn_fwd_args, workspace) P(ltxattn_fwd_args, num_splits)
  P(ltxattn_fwd_args, causal) P(ltxattn_fwd_args, window) P(ltxattn_fwd_args, kv_heads)
  P(ltxattn_fwd_args, gate) P(ltxattn_fwd_args, gate_stride_b) P(ltxattn_fwd_args, gate_stride_h)
  P(ltxattn_fwd_plan_info, units) P(ltxattn_fwd_plan_info, split_units) P(ltxattn_fwd_plan_info, launches)
  P(ltxattn_bwd_args, dout) P(ltxattn_bwd_args, lse) P(ltxattn_bwd_args, dq) P(ltxattn_bwd_args, scale)
  P(ltxattn_bwd_args, k_rotary) P(ltxattn_bwd_args, workspace_bytes)
  P(ltxattn_rotary, tokens) P(ltxattn_device_info, total_memory_bytes) P(ltxattn_device_info, supported)
  P(ltxattn_rope_args, x) P(ltxattn_rope_args, out) P(ltxattn_rope_args, rotary)
  P(ltxattn_rotary_table_args, theta) P(ltxattn_rotary_table_args, max_pos) P(ltxattn_rotary_table_args, positions)
  P(ltxattn_rotary_table_args, sin)
  P(ltxattn_qk_prep_args, x) P(ltxattn_qk_prep_args, weight) P(ltxattn_qk_prep_args, eps)
  P(ltxattn_qk_prep_args, rotary) P(ltxattn_qk_prep_args, out)
  return 0;
}
"""


def test_ctypes_layout_matches_the_header(tmp_path):
    src = tmp_path / "probe.c"
    src.write_text(PROBE)
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-std=c11", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = dict(ln.rsplit(" ", 1) for ln in subprocess.run([str(exe)], capture_output=True, text=True,
                                                         check=True).stdout.splitlines())
    sizes = {"ltxattn_tensor": _lib.Tensor, "ltxattn_rotary": _lib.Rotary, "ltxattn_fwd_args": _lib.FwdArgs,
             "ltxattn_bwd_args": _lib.BwdArgs, "ltxattn_gather_args": _lib.GatherArgs,
             "ltxattn_device_info": _lib.DeviceInfo, "ltxattn_rope_args": _lib.RopeArgs,
             "ltxattn_rotary_table_args": _lib.RotaryTableArgs, "ltxattn_qk_prep_args": _lib.QkPrepArgs,
             "ltxattn_fwd_plan_info": _lib.FwdPlanInfo, "ltxattn_memory_plan_args": _lib.MemoryPlanArgs,
             "ltxattn_memory_plan_info": _lib.MemoryPlanInfo, "ltxattn_linear_args": _lib.LinearArgs,
             "ltxattn_out_project_args": _lib.OutProjectArgs, "ltxattn_head_gate_args": _lib.HeadGateArgs,
             "ltxattn_gather_peers": _lib.GatherPeers, "ltxattn_reduce_peers": _lib.ReducePeers}
    for cname, py in sizes.items():
        assert int(got[cname]) == ctypes.sizeof(py), cname
    structs = {"ltxattn_fwd_args": _lib.FwdArgs, "ltxattn_bwd_args": _lib.BwdArgs,
               "ltxattn_rotary": _lib.Rotary, "ltxattn_device_info": _lib.DeviceInfo,
               "ltxattn_rope_args": _lib.RopeArgs, "ltxattn_rotary_table_args": _lib.RotaryTableArgs,
               "ltxattn_qk_prep_args": _lib.QkPrepArgs, "ltxattn_fwd_plan_info": _lib.FwdPlanInfo,
               "ltxattn_memory_plan_args": _lib.MemoryPlanArgs, "ltxattn_memory_plan_info": _lib.MemoryPlanInfo,
               "ltxattn_linear_args": _lib.LinearArgs, "ltxattn_out_project_args": _lib.OutProjectArgs,
               "ltxattn_head_gate_args": _lib.HeadGateArgs, "ltxattn_gather_peers": _lib.GatherPeers,
               "ltxattn_reduce_peers": _lib.ReducePeers}
    for key, val in got.items():
        if "." in key:
            s, f = key.split(".")
            assert getattr(structs[s], f).offset == int(val), key


def _args(**kw):
    a = _lib.FwdArgs()
    a.dtype, a.batch, a.heads, a.q_len, a.kv_len, a.head_dim = _lib.BF16, 1, 2, 16, 16, 64
    for k, v in kw.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("kw,status", [
    (dict(dtype=7), _lib.ERR_DTYPE),
    (dict(head_dim=80), _lib.ERR_UNSUPPORTED),
    (dict(head_dim=256), _lib.ERR_UNSUPPORTED),
    (dict(batch=0), _lib.ERR_SHAPE),
    (dict(kv_len=0), _lib.ERR_SHAPE),
    (dict(head_begin=1, head_count=2), _lib.ERR_ARG),
    (dict(kv_len=200000), _lib.ERR_UNSUPPORTED),
    (dict(causal=1, kv_len=32), _lib.ERR_SHAPE),      # causal needs q_len == kv_len
    (dict(kv_heads=3), _lib.ERR_SHAPE),               # kv_heads must divide heads
    (dict(window=-1), _lib.ERR_ARG),
])
def test_validation_refuses_before_any_device_work(kw, status):
    L = _lib.load()
    rc = L.ltxattn_fwd(ctypes.byref(_args(**kw)), None)
    assert rc == status, (_lib.last_error(), rc)
    assert _lib.last_error() != ""
    assert L.ltxattn_fwd_workspace(ctypes.byref(_args(**kw))) == 0


def test_null_arguments():
    L = _lib.load()
    assert L.ltxattn_fwd(None, None) == _lib.ERR_ARG
    assert L.ltxattn_device_count(None) == _lib.ERR_ARG
    assert L.ltxattn_device_query(0, None) == _lib.ERR_ARG
    assert L.ltxattn_allgather_heads(None, None, None) == _lib.ERR_ARG
    assert L.ltxattn_comm_destroy(None) == _lib.OK


def test_rotary_table_must_cover_the_tokens():
    L = _lib.load()
    a = _args()
    a.q_rotary = _lib.Rotary(cos=1024, sin=2048, stride_b=0, stride_h=0, stride_t=32, tokens=8)
    assert L.ltxattn_fwd(ctypes.byref(a), None) == _lib.ERR_SHAPE
    assert "q_rotary covers 8 tokens" in _lib.last_error()


def test_variant_rotary_rule_mirrors_the_reference():
    # DiTAttention.swift:319-321: attn2 / audio_attn2 take no rotary embedding
    assert not backend.Variant.video_cross.takes_rotary
    assert not backend.Variant.audio_cross.takes_rotary
    assert backend.Variant.audio_to_video.takes_rotary
    e = backend.Failure.rotary_without_position(backend.Variant.video_cross)
    assert e.kind == "rotaryWithoutPosition" and "attn2 takes no rotary" in str(e)
    assert str(backend.Failure.shape("q", (1, 2), "[B, H, T, D]")) == "q is [1, 2], expected [B, H, T, D]"


def test_grouped_kv_heads_take_no_rotary():
    # grouped KV heads (the Gemma encoder) rotate before the call (GemmaTextEncoder.swift:173,193)
    L = _lib.load()
    a = _args(heads=4, kv_heads=2)
    a.q_rotary = _lib.Rotary(cos=1024, sin=2048, stride_b=0, stride_h=0, stride_t=32, tokens=16)
    assert L.ltxattn_fwd(ctypes.byref(a), None) == _lib.ERR_UNSUPPORTED
    assert "grouped KV heads" in _lib.last_error()


@pytest.mark.parametrize("shape,want", [
    # (B, H, Lq, Lk, D), (kernel, splits, split_units, launches); 148 SMs (no device here)
    ((1, 32, 3120, 3120, 128), (1, 1, 0, 1)),     # config 2: 416 units, one CTA each
    ((1, 32, 3120, 512, 128), (3, 1, 0, 1)),      # 4 KV tiles: the persistent kernel's cheaper unit boundary wins
    ((1, 32, 29760, 29760, 128), (1, 3, 44, 2)),  # config 5 on 1 GPU: 25 waves + 44 units split 3 ways
    ((1, 32, 3120, 1024, 128, "mask"), (3, 1, 0, 1)),  # config 3: masked, 416 units, persistent
    ((1, 32, 3120, 126, 64), (2, 1, 0, 1)),       # config 4b: one KV tile -> persistent kernel
    ((1, 32, 126, 3120, 64), (1, 4, 32, 2)),      # config 4c: one wave of 4-way splits + combine
    ((1, 4, 29760, 29760, 128), (1, 6, 24, 2)),   # config 5 on 8 GPUs: the last 24 units split 6 ways
    ((1, 32, 126, 126, 64), (1, 1, 0, 1)),        # config 4a: 32 units, one KV tile, nothing to split
])
def test_forward_plan(shape, want):
    B, H, Lq, Lk, D = shape[:5]
    a = _lib.FwdArgs()
    a.dtype, a.batch, a.heads, a.q_len, a.kv_len, a.head_dim = _lib.BF16, B, H, Lq, Lk, D
    if "mask" in shape:
        a.key_mask, a.key_mask_stride_b = 4096, Lk
    info = _lib.FwdPlanInfo()
    assert _lib.load().ltxattn_fwd_plan(ctypes.byref(a), ctypes.byref(info)) == _lib.OK, _lib.last_error()
    assert (info.kernel, info.splits, info.split_units, info.launches) == want
    a.dtype = _lib.F32
    assert _lib.load().ltxattn_fwd_plan(ctypes.byref(a), ctypes.byref(info)) == _lib.OK
    assert info.kernel == 0 and info.splits == 1


def test_gate_strides_must_be_non_negative():
    L = _lib.load()
    a = _args()
    for name in ("q", "k", "v", "out"):
        setattr(a, name, _lib.Tensor(data=4096, stride_b=2 * 16 * 64, stride_h=16 * 64, stride_t=64))
    a.gate, a.gate_stride_b, a.gate_stride_t, a.gate_stride_h = 8192, 32, 2, -1
    assert L.ltxattn_fwd(ctypes.byref(a), None) == _lib.ERR_SHAPE
    assert "gate has a negative stride" in _lib.last_error()


def test_new_entry_points_refuse_bad_arguments():
    L = _lib.load()
    assert L.ltxattn_rope(None, None) == _lib.ERR_ARG
    assert L.ltxattn_rotary_tables(None, None) == _lib.ERR_ARG
    assert L.ltxattn_qk_prep(None, None) == _lib.ERR_ARG
    r = _lib.RopeArgs()
    r.dtype, r.batch, r.heads, r.tokens, r.head_dim = _lib.BF16, 1, 1, 4, 64
    assert L.ltxattn_rope(ctypes.byref(r), None) == _lib.ERR_ARG  # no tables
    t = _lib.RotaryTableArgs()
    t.dtype, t.n_pos, t.tokens, t.inner, t.heads, t.theta = _lib.BF16, 5, 4, 4096, 32, 10000.0
    assert L.ltxattn_rotary_tables(ctypes.byref(t), None) == _lib.ERR_SHAPE  # n_pos > 4
    q = _lib.QkPrepArgs()
    q.dtype, q.batch, q.tokens, q.heads, q.head_dim = _lib.BF16, 1, 4, 3, 64  # inner 192
    assert L.ltxattn_qk_prep(ctypes.byref(q), None) == _lib.ERR_UNSUPPORTED


def test_selftest_and_comm_size_refuse_bad_arguments():
    # argument checks that run before any device work
    L = _lib.load()
    assert L.ltxattn_selftest_wait_timeout(0, None) == _lib.ERR_ARG
    assert L.ltxattn_selftest_wait_timeout(1000001, None) == _lib.ERR_ARG
    assert "limit_us" in _lib.last_error()
    n = ctypes.c_int32()
    assert L.ltxattn_comm_size(None, ctypes.byref(n), ctypes.byref(n)) == _lib.ERR_ARG


def test_memory_plan_counts_the_call_buffers():
    # config 2 (3120 tokens, 32 heads of 128, bf16, rotary): q, k, v, out are 25.6 MB
    # each, lse 0.4 MB, and the rotated q / k copies in the workspace another 2 x 25.6 MB
    L = _lib.load()
    a = _lib.MemoryPlanArgs(dtype=_lib.BF16, batch=1, heads=32, tokens=3120, head_dim=128, rotary=1,
                            training=0, resident_bytes=42_060_000_000, available_bytes=180_000_000_000,
                            margin_fraction=0.15)
    info = _lib.MemoryPlanInfo()
    assert L.ltxattn_memory_plan(ctypes.byref(a), ctypes.byref(info)) == _lib.OK, _lib.last_error()
    act = 3120 * 32 * 128 * 2
    assert info.tensor_bytes == 4 * act + 3120 * 32 * 4
    assert info.workspace_bytes >= 2 * act  # rotated q and k
    assert info.backward_bytes == 0
    assert info.peak_bytes == 42_060_000_000 + info.tensor_bytes + info.workspace_bytes
    want_headroom = 180_000_000_000 - round(info.peak_bytes * 1.15)
    assert info.headroom_bytes == want_headroom and info.fits == 1
    assert abs(info.bytes_per_token * 3120 - (info.tensor_bytes + info.workspace_bytes)) < 1.0
    # training adds dout, dq, dk, dv and the backward's workspace
    a.training = 1
    t = _lib.MemoryPlanInfo()
    assert L.ltxattn_memory_plan(ctypes.byref(a), ctypes.byref(t)) == _lib.OK
    assert t.backward_bytes >= 4 * act
    # a device too small for the resident weights does not fit
    a.available_bytes = 40_000_000_000
    assert L.ltxattn_memory_plan(ctypes.byref(a), ctypes.byref(t)) == _lib.OK and t.fits == 0
    # refusals
    a.head_dim = 80
    assert L.ltxattn_memory_plan(ctypes.byref(a), ctypes.byref(t)) == _lib.ERR_UNSUPPORTED
    a.head_dim, a.margin_fraction = 128, -0.1
    assert L.ltxattn_memory_plan(ctypes.byref(a), ctypes.byref(t)) == _lib.ERR_ARG
    assert L.ltxattn_memory_plan(None, ctypes.byref(t)) == _lib.ERR_ARG


def test_linear_plans_split_k_for_narrow_outputs_only():
    # 32 gate logits of 3120 rows: 25 tiles fill few SMs, so a workspace for K
    # splits is asked for; a 4096-wide projection fills the GPU and asks for none
    L = _lib.load()
    a = _lib.LinearArgs(dtype=_lib.BF16, m=3120, n=32, k=4096)
    need = L.ltxattn_linear_workspace(ctypes.byref(a))
    assert need > 0 and need % 256 == 0 and need >= 2 * 3120 * 32 * 4
    a.n = 4096
    assert L.ltxattn_linear_workspace(ctypes.byref(a)) == 0
    a.n, a.k = 32, 192  # too short a K to split
    assert L.ltxattn_linear_workspace(ctypes.byref(a)) == 0


def _peers(world=2, rank=0, epoch=1, out=None):
    g = _lib.GatherPeers()
    g.world, g.rank, g.epoch = world, rank, epoch
    for d in range(8):
        g.out[d] = 4096 * (d + 1)
        g.signals[d] = 4096 * (d + 9)
    if out is not None:
        g.out[rank] = out
    return g


@pytest.mark.parametrize("kw,peers,status", [
    (dict(dtype=_lib.F32), dict(), _lib.ERR_DTYPE),
    (dict(), dict(world=1), _lib.ERR_ARG),           # 2 to 8 ranks
    (dict(), dict(world=9), _lib.ERR_ARG),
    (dict(), dict(rank=2), _lib.ERR_ARG),            # rank outside the world
    (dict(), dict(epoch=0), _lib.ERR_ARG),           # epochs start at 1
    (dict(), dict(out=8192), _lib.ERR_ARG),          # peers.out[rank] must be args.out
])
def test_fused_gather_validation_refuses_before_any_device_work(kw, peers, status):
    # ltxattn_fwd_gather checks its peer description on the host first
    L = _lib.load()
    a = _args(**kw)
    a.out.data = 4096  # == _peers().out[0]
    rc = L.ltxattn_fwd_gather(ctypes.byref(a), ctypes.byref(_peers(**peers)), None)
    assert rc == status, (_lib.last_error(), rc)
    assert "ltxattn_fwd_gather" in _lib.last_error()


def test_fused_gather_refuses_unaligned_peer_outputs():
    L = _lib.load()
    a = _args()
    a.out.data = 4096
    g = _peers()
    g.out[1] = 4096 * 2 + 8  # rank 1's output not 16-byte aligned
    assert L.ltxattn_fwd_gather(ctypes.byref(a), ctypes.byref(g), None) == _lib.ERR_ALIGN


def _reduce_peers(world=2, rank=0, epoch=1):
    g = _lib.ReducePeers()
    g.world, g.rank, g.epoch = world, rank, epoch
    for d in range(8):
        g.recv[d] = 4096 * (d + 1)
        g.out[d] = 4096 * (d + 17)
        g.signals[d] = 4096 * (d + 33)
    return g


@pytest.mark.parametrize("field,value,peers,status", [
    ("dtype", _lib.F32, dict(), _lib.ERR_DTYPE),
    ("n", 12, dict(), _lib.ERR_SHAPE),               # n a multiple of 8
    ("m", 0, dict(), _lib.ERR_SHAPE),
    (None, None, dict(world=1), _lib.ERR_ARG),
    (None, None, dict(rank=5), _lib.ERR_ARG),
    (None, None, dict(epoch=0), _lib.ERR_ARG),
    ("out", 8192, dict(), _lib.ERR_ARG),             # peers.out[rank] must be args.out
])
def test_fused_out_project_validation_refuses_before_any_device_work(field, value, peers, status):
    L = _lib.load()
    a = _lib.OutProjectArgs()
    a.dtype, a.m, a.n, a.k = _lib.BF16, 300, 512, 1024
    a.out, a.out_stride = 4096 * 17, 512
    if field is not None:
        setattr(a, field, value)
    rc = L.ltxattn_out_project_fused(ctypes.byref(a), ctypes.byref(_reduce_peers(**peers)), None)
    assert rc == status, (_lib.last_error(), rc)
    assert "ltxattn_out_project_fused" in _lib.last_error()
