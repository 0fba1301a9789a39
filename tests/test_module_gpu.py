"""A whole DiT attention module (DiTAttention.callAsFunction,
DiTAttention.swift:315-404) on the device -- every step in libltxattn_cuda
(tcgen05 projections with the norms, split and RoPE fused into the q / k
projection, the attention, the gate and the merge), and the same module with
the projections on torch's library GEMM -- against the CPU oracle's
composition of the same steps (``oracle.dit_attention_module``).

Tolerance: the bf16 bar (max abs <= 2e-2, rel-L2 <= 1e-2) on the module output;
the projections' fp32-accumulated GEMMs and the oracle's fp64 ones may round a
bf16 value differently, which the later steps carry along.
"""
import numpy as np
import pytest
import torch

import oracle
from ltxattn import DiTAttentionModule, Failure, Rotary, Variant, inputs

pytestmark = pytest.mark.gpu


def weights(seed, query_dim, inner, kv_dim, gate, heads):
    rng = np.random.default_rng(seed)
    def mat(o, i):
        return inputs.round_bf16(rng.normal(0.0, 1.0 / np.sqrt(i), (o, i)).astype(np.float32))
    def vec(n, lo=-0.1, hi=0.1):
        return inputs.round_bf16(rng.uniform(lo, hi, n).astype(np.float32))
    w = {"to_q.weight": mat(inner, query_dim), "to_q.bias": vec(inner),
         "to_k.weight": mat(inner, kv_dim), "to_k.bias": vec(inner),
         "to_v.weight": mat(inner, kv_dim), "to_v.bias": vec(inner),
         "to_out.0.weight": mat(query_dim, inner), "to_out.0.bias": vec(query_dim),
         "q_norm.weight": vec(inner, 0.5, 1.5), "k_norm.weight": vec(inner, 0.5, 1.5)}
    if gate:
        w["to_gate_logits.weight"] = mat(heads, query_dim)
        w["to_gate_logits.bias"] = vec(heads)
    return w


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda", torch.bfloat16)


def check(got, want, what):
    g = got.float().cpu().numpy().astype(np.float64)
    err = np.abs(g - want)
    rel = np.linalg.norm(err) / np.linalg.norm(want)
    assert err.max() <= 2e-2 and rel <= 1e-2, f"{what}: max abs {err.max():.3e} rel-L2 {rel:.3e}"


@pytest.mark.parametrize("gemm", ["ltxattn", "torch"])
@pytest.mark.parametrize("gate", [True, False])
def test_video_self_attention_module(gate, gemm):
    B, T, heads, D = 1, 96, 8, 64
    inner = query_dim = heads * D
    w = weights(3, query_dim, inner, query_dim, gate, heads)
    x = inputs.round_bf16(inputs.seeded_tensor(5, (B, T, query_dim)))
    cos, sin = inputs.rope1d(np.arange(T, dtype=np.float64), D)
    want = oracle.dit_attention_module(x, w, heads, cos, sin)
    mod = DiTAttentionModule({k: dev(v) for k, v in w.items()}, heads, gemm=gemm)
    got = mod(dev(x), rotary=Rotary(dev(cos), dev(sin)))
    check(got, want, f"self gate={gate} gemm={gemm}")


def test_cross_modal_module_with_separate_key_tables():
    # audio_to_video_attn: queries from the video stream, keys/values from audio,
    # separate key positions (DiTAttention.swift:309-314)
    B, T, Tk, heads, D = 1, 80, 40, 8, 64
    inner = heads * D
    query_dim, kv_dim = 1024, inner
    w = weights(7, query_dim, inner, kv_dim, True, heads)
    x = inputs.round_bf16(inputs.seeded_tensor(8, (B, T, query_dim)))
    ctx = inputs.round_bf16(inputs.seeded_tensor(9, (B, Tk, kv_dim)))
    qc, qs = inputs.rope1d(np.arange(T, dtype=np.float64) * 0.25, D)
    kc, ks = inputs.rope1d(np.arange(Tk, dtype=np.float64) * 0.5, D)
    want = oracle.dit_attention_module(x, w, heads, qc, qs, kc, ks, context=ctx)
    mod = DiTAttentionModule({k: dev(v) for k, v in w.items()}, heads, Variant.audio_to_video)
    got = mod(dev(x), context=dev(ctx), rotary=Rotary(dev(qc), dev(qs)), key_rotary=Rotary(dev(kc), dev(ks)))
    check(got, want, "cross-modal")


def test_text_cross_attention_takes_no_rotary():
    heads, D = 8, 64
    w = weights(11, heads * D, heads * D, heads * D, False, heads)
    mod = DiTAttentionModule({k: dev(v) for k, v in w.items()}, heads, Variant.video_cross)
    x = torch.zeros((1, 16, heads * D), device="cuda", dtype=torch.bfloat16)
    cos = torch.ones((16, D // 2), device="cuda", dtype=torch.bfloat16)
    with pytest.raises(Failure):
        mod(x, rotary=Rotary(cos, cos))


@pytest.mark.parametrize("gate", [True, False])
def test_stg_passthrough_gates_and_merges_the_value_stream(gate):
    # all_perturbed (DiTAttention.swift:349-356): v, split, gated (ltxattn_head_gate), merged, to_out
    B, T, heads, D = 1, 96, 8, 64
    inner = query_dim = heads * D
    w = weights(13, query_dim, inner, query_dim, gate, heads)
    x = inputs.round_bf16(inputs.seeded_tensor(14, (B, T, query_dim)))
    v = oracle.linear(x, w["to_v.weight"], w["to_v.bias"])
    vh = v.reshape(B, T, heads, D).transpose(0, 2, 1, 3)
    if gate:
        vh = oracle.gate_output(vh, oracle.linear(x, w["to_gate_logits.weight"], w["to_gate_logits.bias"]))
    merged = np.ascontiguousarray(vh.transpose(0, 2, 1, 3).reshape(B, T, inner))
    want = oracle.linear(merged, w["to_out.0.weight"], w["to_out.0.bias"])
    mod = DiTAttentionModule({k: dev(v) for k, v in w.items()}, heads)
    got = mod(dev(x), all_perturbed=True)
    check(got, want, f"passthrough gate={gate}")
