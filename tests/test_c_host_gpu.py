"""The C ABI from a plain C host, the way the Swift shim binds it.

tests/c/abi_host.c includes only include/ltxattn.h and the CUDA runtime: it
queries the device (ltxattn_device_count / ltxattn_device_query, the
LTXHardware.Machine replacement), runs one bf16 forward with split RoPE and
the log-sum-exp (ltxattn_fwd) and its backward (ltxattn_bwd) on the reference
bench's operand stream, checks the device error word, and writes every input
and output to a file.  The program is built here with gcc (a CPU test); on a
GPU it runs and its results are checked against the CPU oracle.
"""
import os
import subprocess

import numpy as np
import pytest

import oracle
from ltxattn import inputs

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "ltx-2.5-swift_b200")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def build(tmp_path):
    exe = tmp_path / "abi_host"
    cmd = ["gcc", "-std=c11", "-O2", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(CUDA, "include"), os.path.join(ROOT, "tests", "c", "abi_host.c"),
           "-L", PKG, "-lltxattn_cuda", "-L", os.path.join(CUDA, "lib64"), "-lcudart", "-lm",
           f"-Wl,-rpath,{PKG}:{os.path.join(CUDA, 'lib64')}", "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def test_c_host_program_builds_against_the_header(tmp_path):
    exe = build(tmp_path)
    assert exe.exists()


def _bf16(bits):
    return inputs.bf16_to_f32(bits)


@pytest.mark.gpu
def test_c_host_forward_and_backward_match_the_oracle(tmp_path):
    exe = build(tmp_path)
    out_file = tmp_path / "abi_host.bin"
    r = subprocess.run([str(exe), str(out_file)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    raw = out_file.read_bytes()
    assert raw[:4] == b"LTXA"
    B, H, T, D = (int(x) for x in np.frombuffer(raw[4:20], np.int32))
    n, nt, nl = B * H * T * D, T * (D // 2), B * H * T
    off = 20

    def take(count, dt):
        nonlocal off
        a = np.frombuffer(raw, dt, count, off)
        off += count * np.dtype(dt).itemsize
        return a
    shp = (B, H, T, D)
    q, k, v = (_bf16(take(n, np.uint16)).reshape(shp) for _ in range(3))
    cos, sin = (_bf16(take(nt, np.uint16)).reshape(1, 1, T, D // 2) for _ in range(2))
    out = _bf16(take(n, np.uint16)).reshape(shp)
    lse = take(nl, np.float32).reshape(B, H, T)
    do = _bf16(take(n, np.uint16)).reshape(shp)
    dq, dk, dv = (_bf16(take(n, np.uint16)).reshape(shp) for _ in range(3))
    assert off == len(raw)
    # the operands are the reference bench's stream (the C restatement agrees with ltxattn.inputs)
    assert np.array_equal(q.ravel(), inputs.bench_bits(0x5EED + 2, n))

    ref, ref_lse = oracle.attention_reference(q, k, v, q_rot=(cos, sin), bf16=True)
    err = np.abs(out - ref)
    assert err.max() <= 2e-2 and np.linalg.norm(err) / np.linalg.norm(ref) <= 1e-2
    assert np.abs(lse - ref_lse).max() < 2e-3

    qr, kr = oracle.rope(q, cos, sin, True), oracle.rope(k, cos, sin, True)
    rq, rk, rv = oracle.attn_bwd(qr, kr, v, do)
    rq, rk = oracle.rope_bwd(rq, cos, sin, True), oracle.rope_bwd(rk, cos, sin, True)
    for name, g, ref_g in (("dq", dq, rq), ("dk", dk, rk), ("dv", dv, rv)):
        e = np.abs(g.astype(np.float64) - ref_g)
        scale = max(1.0, float(np.abs(ref_g).max()))
        rel = np.linalg.norm(e) / max(np.linalg.norm(ref_g), 1e-3 * np.sqrt(ref_g.size))
        assert e.max() <= 2e-2 * scale and rel <= 1e-2, (name, e.max(), rel)
