"""The library inside CUDA graphs: the forward call (RoPE pre-pass, attention
kernel launched with programmatic stream serialization, split combine), the
persistent one-tile kernel, a whole attention module and the backward are
captured once and replayed; every replay must reproduce the eager result bit
for bit.  (Argument validation, tensor maps and workspace are set up before
capture; a call makes no allocation of its own.)
"""
import numpy as np
import pytest
import torch

from ltxattn import AttentionBackend, DiTAttentionModule, Rotary, device_status, inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def no_kernel_timeouts():
    yield
    assert device_status(clear=True) == 0, "a kernel wait timed out"


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda", torch.bfloat16)


def same_bits(a, b):
    return torch.equal(a.contiguous().view(torch.int16), b.contiguous().view(torch.int16))


def capture(fn):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()  # warm-up on the capture stream (one-time kernel attributes, allocator)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g


@pytest.mark.parametrize("shape", [(1, 8, 126, 3120, 64), (1, 32, 3120, 126, 64), (1, 4, 700, 900, 128)])
def test_forward_call_replays_in_a_graph(shape):
    B, H, Lq, Lk, D = shape
    q = dev(inputs.seeded_tensor(3, (B, H, Lq, D), rmsnorm=True))
    k = dev(inputs.seeded_tensor(4, (B, H, Lk, D), rmsnorm=True))
    v = dev(inputs.seeded_tensor(5, (B, H, Lk, D)))
    qc, qs = inputs.rope1d(np.arange(Lq, dtype=np.float64) * 0.5, D)
    kc, ks = inputs.rope1d(np.arange(Lk, dtype=np.float64) * 0.25, D)
    prep = AttentionBackend.prepare(q, k, v, q_rotary=Rotary(dev(qc), dev(qs)), k_rotary=Rotary(dev(kc), dev(ks)),
                                    save_lse=True)
    eager_out, eager_lse = [t.clone() for t in prep.run()]
    prep.out.zero_()
    g = capture(lambda: prep.run(torch.cuda.current_stream()))
    for _ in range(3):
        prep.out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert same_bits(prep.out, eager_out) and torch.equal(prep.lse, eager_lse)


def test_module_and_backward_replay_in_graphs():
    B, T, heads, D = 1, 512, 8, 64
    dim = heads * D
    rng = np.random.default_rng(2)
    w = {n: dev(rng.normal(0, 1 / np.sqrt(dim), (dim, dim)).astype(np.float32)) for n in
         ("to_q.weight", "to_k.weight", "to_v.weight", "to_out.0.weight")}
    w.update({"q_norm.weight": dev(np.ones(dim, np.float32)), "k_norm.weight": dev(np.ones(dim, np.float32)),
              "to_gate_logits.weight": dev(rng.normal(0, 0.05, (heads, dim)).astype(np.float32))})
    mod = DiTAttentionModule(w, heads)
    x = dev(inputs.seeded_tensor(9, (B, T, dim)))
    c, s = inputs.rope1d(np.arange(T, dtype=np.float64), D)
    rot = Rotary(dev(c), dev(s))
    eager = mod(x, rotary=rot).clone()
    out = {}
    g = capture(lambda: out.__setitem__("y", mod(x, rotary=rot)))
    g.replay()
    torch.cuda.synchronize()
    assert same_bits(out["y"], eager)

    q = dev(inputs.seeded_tensor(11, (1, 4, 1000, 128), rmsnorm=True))
    k = dev(inputs.seeded_tensor(12, (1, 4, 1000, 128), rmsnorm=True))
    v = dev(inputs.seeded_tensor(13, (1, 4, 1000, 128)))
    do = dev(inputs.seeded_tensor(14, (1, 4, 1000, 128)))
    o, lse = AttentionBackend.attention(q, k, v, save_lse=True)
    ref = [t.clone() for t in AttentionBackend.attention_backward(q, k, v, o, do, lse)]
    grads = [torch.empty_like(t) for t in (q, k, v)]
    g2 = capture(lambda: AttentionBackend.attention_backward(q, k, v, o, do, lse, dq=grads[0], dk=grads[1], dv=grads[2]))
    for t in grads:
        t.zero_()
    g2.replay()
    torch.cuda.synchronize()
    assert all(same_bits(a, b) for a, b in zip(grads, ref))
