"""Host-side fuzzing of the forward planner (no GPU): random shapes, split
requests and masks through ltxattn_fwd_plan / ltxattn_fwd_workspace must never
crash and must stay self-consistent -- a split plan always has scratch for its
partials, every launch fits the 1-D grid, and the persistent kernel is chosen
only for one-tile key sequences (kernel 2) or for unbanded calls of at least a
wave of units (kernel 3).  148 SMs are assumed (no device here)."""
import ctypes

from hypothesis import given, settings, strategies as st

from ltxattn import _lib

KMAX_SPLITS = 32


@settings(max_examples=400, deadline=None)
@given(B=st.integers(1, 4), H=st.integers(1, 96), Lq=st.integers(1, 40000), Lk=st.integers(1, 40000),
       D=st.sampled_from([64, 128]), splits=st.integers(0, 40), masked=st.booleans(),
       causal=st.booleans(), window=st.integers(0, 600), bf16=st.booleans())
def test_plan_is_self_consistent(B, H, Lq, Lk, D, splits, masked, causal, window, bf16):
    L = _lib.load()
    a = _lib.FwdArgs()
    a.dtype = _lib.BF16 if bf16 else _lib.F32
    a.batch, a.heads, a.q_len, a.kv_len, a.head_dim = B, H, Lq, (Lq if causal else Lk), D
    a.num_splits = splits
    a.causal, a.window = int(causal), window
    if masked:
        a.key_mask, a.key_mask_stride_b = 4096, a.kv_len
    info = _lib.FwdPlanInfo()
    rc = L.ltxattn_fwd_plan(ctypes.byref(a), ctypes.byref(info))
    ws = L.ltxattn_fwd_workspace(ctypes.byref(a))
    if rc != _lib.OK:
        assert ws == 0
        return
    kv_tiles = (a.kv_len + 127) // 128
    if not bf16:
        assert info.kernel == 0 and info.splits == 1 and ws == 0
        return
    q_blocks = (Lq + 255) // 256
    assert info.units == q_blocks * H * B
    assert 1 <= info.splits <= min(KMAX_SPLITS, kv_tiles) or (info.splits == 1)
    assert 0 <= info.split_units <= info.units
    if info.splits > 1:
        assert info.split_units > 0 and ws > 0 and info.launches == 2
        # partials: splits x split units x 256 rows x (D + 1) floats
        assert ws >= info.splits * info.split_units * 256 * (D + 1) * 4
    else:
        assert info.split_units == 0 and ws == 0 and info.launches == 1
    if info.kernel == 2:
        assert kv_tiles == 1 and not causal and window == 0 and splits == 0 and info.units > 148
    if info.kernel == 3:  # persistent whole units: unbanded, at least a wave, more than one KV tile
        assert not causal and window == 0 and splits == 0
        assert info.units >= 148 and kv_tiles > 1 and info.splits == 1 and info.launches == 1
    assert info.units - info.split_units + info.split_units * info.splits < 2 ** 31
