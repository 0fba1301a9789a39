"""The Gemma text encoder's self-attention on a B200 (GemmaTextEncoder.swift:
218-233, 292-323): causal and sliding-window masks, key padding with the
un-masking of rows left without keys, grouped KV heads -- against the fp64 CPU
oracle.  Tolerances as for the DiT attention: fp32 max abs <= 1e-5; bf16 max
abs <= 2e-2 and rel-L2 <= 1e-2; LSE within 2e-3.
"""
import numpy as np
import pytest
import torch

import oracle
from ltxattn import AttentionBackend, device_status, inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def no_kernel_timeouts():
    yield
    assert device_status(clear=True) == 0, "a kernel wait timed out"


def run_case(dtype, B, Hq, Hkv, L, D, causal, window, pad, scale, seed=51, empty_batch=None):
    bf = dtype == torch.bfloat16
    q = inputs.seeded_tensor(seed + 2, (B, Hq, L, D), rmsnorm=True, bf16=bf)
    k = inputs.seeded_tensor(seed + 3, (B, Hkv, L, D), rmsnorm=True, bf16=bf)
    v = inputs.seeded_tensor(seed + 4, (B, Hkv, L, D), bf16=bf)
    valid = np.ones((B, L), np.uint8)
    if pad:
        valid[:, :pad] = 0  # left padding: the first rows have no valid key at or before them
    if empty_batch is not None:
        valid[empty_batch] = 0
    want, want_lse = oracle.attention_gemma(q, k, v, valid, scale, causal, window)
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dtype)
    out, lse = AttentionBackend.attention(dev(q), dev(k), dev(v), scale,
                                          key_mask=torch.from_numpy(valid.astype(bool)).cuda(),
                                          save_lse=True, causal=causal, window=window)
    torch.cuda.synchronize()
    g = out.float().cpu().numpy().astype(np.float64)
    err = np.abs(g - want)
    if dtype == torch.float32:
        assert err.max() <= 1e-5, f"max abs {err.max():.3e}"
    else:
        rel = np.linalg.norm(err) / np.linalg.norm(want)
        assert err.max() <= 2e-2 and rel <= 1e-2, f"max abs {err.max():.3e} rel-L2 {rel:.3e}"
    lerr = np.abs(lse.cpu().numpy() - want_lse).max()
    assert lerr <= 2e-3, f"lse max abs {lerr:.3e}"


@pytest.mark.parametrize("dtype,B,Hq,Hkv,L,D,causal,window,pad,scale", [
    (torch.bfloat16, 1, 8, 8, 300, 64, True, 0, 0, 0.125),         # full causal layer
    (torch.bfloat16, 2, 8, 2, 330, 128, True, 100, 17, 0.088),     # sliding, left padding, GQA 4:1
    (torch.float32, 1, 4, 1, 200, 64, True, 64, 5, 0.125),         # fp32 parity path
    (torch.bfloat16, 1, 4, 4, 260, 64, True, 0, 0, 1.0),           # Gemma's scale 1.0
])
def test_gemma_attention_matches_oracle(dtype, B, Hq, Hkv, L, D, causal, window, pad, scale):
    run_case(dtype, B, Hq, Hkv, L, D, causal, window, pad, scale)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_batch_without_valid_keys_attends_everything(dtype):
    # batch 1 is all padding: every one of its rows is left without keys and attends all of them
    run_case(dtype, 2, 2, 2, 150, 64, True, 40, 3, 0.125, empty_batch=1)


def test_window_equal_to_length_is_plain_causal():
    # at 1024 tokens a 1024 window coincides with the causal mask (GemmaTextEncoder.swift:289-291)
    run_case(torch.bfloat16, 1, 4, 2, 1024, 128, True, 1024, 9, 0.088)
