"""Device discovery and memory planning on the GPU: ltxattn_device_query and
ltxattn_device_count (the CUDA replacement of LTXHardware.Machine.detect,
Machine.swift:31-36) and ltxattn_memory_plan (the counterpart of
LTXHardware.MemoryPlan, MemoryPlan.swift:27-34,62-74) read from the device
they run on."""
import ctypes

import pytest
import torch

from ltxattn import AttentionBackend, _lib, device_info, qk_prep

pytestmark = pytest.mark.gpu


def test_device_query_describes_the_b200():
    n = ctypes.c_int32()
    assert _lib.load().ltxattn_device_count(ctypes.byref(n)) == _lib.OK
    assert n.value == torch.cuda.device_count() >= 1
    d = device_info(0)
    props = torch.cuda.get_device_properties(0)
    assert (d["cc_major"], d["cc_minor"]) == (props.major, props.minor) == (10, 0)
    assert d["sm_count"] == props.multi_processor_count == 148
    assert d["supported"] == 1
    assert "B200" in d["name"]
    assert abs(d["total_memory_bytes"] - props.total_memory) < (1 << 30)
    assert 0 < d["free_memory_bytes"] <= d["total_memory_bytes"]
    assert d["total_memory_bytes"] > 170e9             # 180 GB of HBM3e
    assert d["l2_bytes"] >= 100 * 1024 * 1024          # 126 MB L2
    assert d["max_smem_per_block_optin"] >= 227 * 1024
    assert d["sm_clock_khz"] > 1_000_000 and d["mem_bus_width_bits"] >= 4096
    # an index past the last device is refused, not read, and the refusal leaves
    # nothing behind: the next launch's error check does not see it
    info = _lib.DeviceInfo()
    assert _lib.load().ltxattn_device_query(n.value, ctypes.byref(info)) != _lib.OK
    q = torch.randn((1, 2, 64, 64), device="cuda").to(torch.bfloat16)
    x = torch.randn((1, 64, 512), device="cuda").to(torch.bfloat16)
    out, _ = AttentionBackend.attention(q, q, q)
    qk_prep(x, torch.ones(512, device="cuda", dtype=torch.bfloat16), 4)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()


def test_memory_plan_reads_the_free_memory_of_the_device():
    a = _lib.MemoryPlanArgs(dtype=_lib.BF16, batch=1, heads=32, tokens=29760, head_dim=128, rotary=0,
                            training=1, resident_bytes=42_060_000_000, available_bytes=0, margin_fraction=0.15)
    info = _lib.MemoryPlanInfo()
    assert _lib.load().ltxattn_memory_plan(ctypes.byref(a), ctypes.byref(info)) == _lib.OK, _lib.last_error()
    free, total = torch.cuda.mem_get_info()
    assert 0 < info.available_bytes <= total
    assert abs(info.available_bytes - free) < (2 << 30)
    # config 5 with its backward next to the reference's 42 GB of DiT weights fits a B200
    assert info.fits == 1 and info.headroom_bytes > 0
    # the counted buffers are what a call at this shape really allocates around the library
    act = 29760 * 32 * 128 * 2
    assert info.tensor_bytes == 4 * act + 29760 * 32 * 4 and info.backward_bytes >= 4 * act
