"""ctypes binding of libltxattn_cuda (include/ltxattn.h).

This is the binding a Python caller of the C ABI uses; the Swift module map in
``swift/`` is the reference-side equivalent.  The library must be the built
in-tree ``libltxattn_cuda.so``: there is no fallback implementation.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(HERE), "libltxattn_cuda.so")

# ltxattn_status
OK, ERR_SHAPE, ERR_DTYPE, ERR_ALIGN, ERR_UNSUPPORTED, ERR_CUDA, ERR_NCCL, ERR_TIMEOUT, ERR_WORKSPACE, \
    ERR_ARG = range(10)
STATUS_NAMES = {OK: "ok", ERR_SHAPE: "shape", ERR_DTYPE: "dtype", ERR_ALIGN: "align",
                ERR_UNSUPPORTED: "unsupported", ERR_CUDA: "cuda", ERR_NCCL: "nccl",
                ERR_TIMEOUT: "timeout", ERR_WORKSPACE: "workspace", ERR_ARG: "arg"}
# ltxattn_dtype
F32, BF16 = 0, 1

EXPORTED = (
    "ltxattn_fwd", "ltxattn_fwd_workspace", "ltxattn_fwd_plan", "ltxattn_fwd_noalloc", "ltxattn_bwd", "ltxattn_bwd_workspace",
    "ltxattn_rope", "ltxattn_rotary_tables", "ltxattn_qk_prep", "ltxattn_qk_prep_pair",
    "ltxattn_comm_unique_id", "ltxattn_comm_init", "ltxattn_comm_destroy",
    "ltxattn_allgather_heads", "ltxattn_device_count", "ltxattn_device_query",
    "ltxattn_last_error", "ltxattn_device_status", "ltxattn_abi_version",
    "ltxattn_comm_size", "ltxattn_selftest_wait_timeout", "ltxattn_memory_plan",
    "ltxattn_linear", "ltxattn_linear_workspace", "ltxattn_head_gate",
    "ltxattn_out_project_workspace", "ltxattn_out_project_allreduce", "ltxattn_fwd_gather",
    "ltxattn_out_project_fused",
)


class Tensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("stride_b", ctypes.c_int64),
                ("stride_h", ctypes.c_int64), ("stride_t", ctypes.c_int64)]


class Rotary(ctypes.Structure):
    _fields_ = [("cos", ctypes.c_void_p), ("sin", ctypes.c_void_p), ("stride_b", ctypes.c_int64),
                ("stride_h", ctypes.c_int64), ("stride_t", ctypes.c_int64),
                ("tokens", ctypes.c_int32)]


class FwdArgs(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int32), ("batch", ctypes.c_int32), ("heads", ctypes.c_int32),
                ("q_len", ctypes.c_int32), ("kv_len", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("head_begin", ctypes.c_int32), ("head_count", ctypes.c_int32),
                ("q", Tensor), ("k", Tensor), ("v", Tensor), ("out", Tensor),
                ("scale", ctypes.c_float), ("key_mask", ctypes.c_void_p),
                ("key_mask_stride_b", ctypes.c_int64), ("q_rotary", Rotary), ("k_rotary", Rotary),
                ("lse", ctypes.c_void_p), ("lse_stride_b", ctypes.c_int64),
                ("lse_stride_h", ctypes.c_int64), ("workspace", ctypes.c_void_p),
                ("workspace_bytes", ctypes.c_size_t), ("num_splits", ctypes.c_int32),
                ("causal", ctypes.c_int32), ("window", ctypes.c_int32), ("kv_heads", ctypes.c_int32),
                ("gate", ctypes.c_void_p), ("gate_stride_b", ctypes.c_int64), ("gate_stride_t", ctypes.c_int64),
                ("gate_stride_h", ctypes.c_int64)]


class GatherPeers(ctypes.Structure):
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("out", ctypes.c_void_p * 8),
                ("signals", ctypes.c_void_p * 8), ("epoch", ctypes.c_uint32), ("reserved", ctypes.c_int32)]


class ReducePeers(ctypes.Structure):
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("recv", ctypes.c_void_p * 8),
                ("out", ctypes.c_void_p * 8), ("signals", ctypes.c_void_p * 8), ("epoch", ctypes.c_uint32),
                ("reserved", ctypes.c_int32)]


class FwdPlanInfo(ctypes.Structure):
    _fields_ = [("kernel", ctypes.c_int32), ("splits", ctypes.c_int32), ("units", ctypes.c_int64),
                ("split_units", ctypes.c_int64), ("launches", ctypes.c_int32)]


class RopeArgs(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int32), ("batch", ctypes.c_int32), ("heads", ctypes.c_int32),
                ("tokens", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("x", Tensor), ("out", Tensor), ("rotary", Rotary)]


class RotaryTableArgs(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int32), ("n_pos", ctypes.c_int32), ("tokens", ctypes.c_int32),
                ("inner", ctypes.c_int32), ("heads", ctypes.c_int32), ("theta", ctypes.c_double),
                ("max_pos", ctypes.c_float * 4), ("positions", ctypes.c_void_p), ("cos", ctypes.c_void_p),
                ("sin", ctypes.c_void_p)]


class QkPrepArgs(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int32), ("batch", ctypes.c_int32), ("tokens", ctypes.c_int32),
                ("heads", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("x", ctypes.c_void_p),
                ("x_stride_b", ctypes.c_int64), ("x_stride_t", ctypes.c_int64), ("weight", ctypes.c_void_p),
                ("eps", ctypes.c_float), ("rotary", Rotary), ("out", Tensor)]


class BwdArgs(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int32), ("batch", ctypes.c_int32), ("heads", ctypes.c_int32),
                ("q_len", ctypes.c_int32), ("kv_len", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("head_begin", ctypes.c_int32), ("head_count", ctypes.c_int32),
                ("q", Tensor), ("k", Tensor), ("v", Tensor), ("out", Tensor), ("dout", Tensor),
                ("lse", ctypes.c_void_p), ("lse_stride_b", ctypes.c_int64),
                ("lse_stride_h", ctypes.c_int64),
                ("dq", Tensor), ("dk", Tensor), ("dv", Tensor),
                ("scale", ctypes.c_float), ("key_mask", ctypes.c_void_p),
                ("key_mask_stride_b", ctypes.c_int64), ("q_rotary", Rotary), ("k_rotary", Rotary),
                ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t)]


class GatherArgs(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int32), ("batch", ctypes.c_int32),
                ("heads_per_rank", ctypes.c_int32), ("tokens", ctypes.c_int32),
                ("head_dim", ctypes.c_int32), ("send", ctypes.c_void_p), ("recv", ctypes.c_void_p)]


class DeviceInfo(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 256), ("device", ctypes.c_int32),
                ("cc_major", ctypes.c_int32), ("cc_minor", ctypes.c_int32),
                ("sm_count", ctypes.c_int32), ("total_memory_bytes", ctypes.c_int64),
                ("free_memory_bytes", ctypes.c_int64), ("max_smem_per_block_optin", ctypes.c_int32),
                ("l2_bytes", ctypes.c_int32), ("sm_clock_khz", ctypes.c_int32),
                ("mem_clock_khz", ctypes.c_int32), ("mem_bus_width_bits", ctypes.c_int32),
                ("supported", ctypes.c_int32)]


_lib = None


class LinearArgs(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int32), ("m", ctypes.c_int32), ("n", ctypes.c_int32), ("k", ctypes.c_int32),
                ("x", ctypes.c_void_p), ("x_stride", ctypes.c_int64), ("weight", ctypes.c_void_p),
                ("weight_stride", ctypes.c_int64), ("bias", ctypes.c_void_p), ("out", ctypes.c_void_p),
                ("out_stride", ctypes.c_int64), ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t)]


class HeadGateArgs(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int32), ("batch", ctypes.c_int32), ("heads", ctypes.c_int32),
                ("tokens", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("x", Tensor), ("out", Tensor),
                ("gate", ctypes.c_void_p), ("gate_stride_b", ctypes.c_int64), ("gate_stride_t", ctypes.c_int64),
                ("gate_stride_h", ctypes.c_int64)]


class OutProjectArgs(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int32), ("m", ctypes.c_int32), ("n", ctypes.c_int32), ("k", ctypes.c_int32),
                ("x", ctypes.c_void_p), ("x_stride", ctypes.c_int64), ("weight", ctypes.c_void_p),
                ("weight_stride", ctypes.c_int64), ("bias", ctypes.c_void_p), ("out", ctypes.c_void_p),
                ("out_stride", ctypes.c_int64), ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t)]


class MemoryPlanArgs(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int32), ("batch", ctypes.c_int32), ("heads", ctypes.c_int32),
                ("tokens", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("rotary", ctypes.c_int32),
                ("training", ctypes.c_int32), ("resident_bytes", ctypes.c_int64),
                ("available_bytes", ctypes.c_int64), ("margin_fraction", ctypes.c_double)]


class MemoryPlanInfo(ctypes.Structure):
    _fields_ = [("tensor_bytes", ctypes.c_int64), ("workspace_bytes", ctypes.c_int64),
                ("backward_bytes", ctypes.c_int64), ("peak_bytes", ctypes.c_int64),
                ("available_bytes", ctypes.c_int64), ("headroom_bytes", ctypes.c_int64),
                ("fits", ctypes.c_int32), ("bytes_per_token", ctypes.c_double)]


def load(path: str = LIB_PATH):
    """Load the in-tree library; raises when it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(
            f"{path} is missing: build it with `python ltx-2.5-swift_b200/build.py` "
            "(there is no CPU fallback)")
    L = ctypes.CDLL(path)
    vp = ctypes.c_void_p
    L.ltxattn_fwd.argtypes = [ctypes.POINTER(FwdArgs), vp]
    L.ltxattn_fwd.restype = ctypes.c_int
    L.ltxattn_fwd_noalloc.argtypes = [ctypes.POINTER(FwdArgs), vp]
    L.ltxattn_fwd_noalloc.restype = ctypes.c_int
    L.ltxattn_fwd_gather.argtypes = [ctypes.POINTER(FwdArgs), ctypes.POINTER(GatherPeers), vp]
    L.ltxattn_fwd_gather.restype = ctypes.c_int
    L.ltxattn_out_project_fused.argtypes = [ctypes.POINTER(OutProjectArgs), ctypes.POINTER(ReducePeers), vp]
    L.ltxattn_out_project_fused.restype = ctypes.c_int
    L.ltxattn_fwd_workspace.argtypes = [ctypes.POINTER(FwdArgs)]
    L.ltxattn_fwd_workspace.restype = ctypes.c_size_t
    L.ltxattn_fwd_plan.argtypes = [ctypes.POINTER(FwdArgs), ctypes.POINTER(FwdPlanInfo)]
    L.ltxattn_fwd_plan.restype = ctypes.c_int
    L.ltxattn_bwd.argtypes = [ctypes.POINTER(BwdArgs), vp]
    L.ltxattn_bwd.restype = ctypes.c_int
    L.ltxattn_bwd_workspace.argtypes = [ctypes.POINTER(BwdArgs)]
    L.ltxattn_bwd_workspace.restype = ctypes.c_size_t
    L.ltxattn_rope.argtypes = [ctypes.POINTER(RopeArgs), vp]
    L.ltxattn_rope.restype = ctypes.c_int
    L.ltxattn_rotary_tables.argtypes = [ctypes.POINTER(RotaryTableArgs), vp]
    L.ltxattn_rotary_tables.restype = ctypes.c_int
    L.ltxattn_qk_prep.argtypes = [ctypes.POINTER(QkPrepArgs), vp]
    L.ltxattn_qk_prep.restype = ctypes.c_int
    L.ltxattn_qk_prep_pair.argtypes = [ctypes.POINTER(QkPrepArgs), ctypes.POINTER(QkPrepArgs), vp]
    L.ltxattn_qk_prep_pair.restype = ctypes.c_int
    L.ltxattn_comm_unique_id.argtypes = [ctypes.POINTER(ctypes.c_uint8)]
    L.ltxattn_comm_unique_id.restype = ctypes.c_int
    L.ltxattn_comm_init.argtypes = [ctypes.POINTER(vp), ctypes.c_int32, ctypes.c_int32,
                                    ctypes.POINTER(ctypes.c_uint8), ctypes.c_int32]
    L.ltxattn_comm_init.restype = ctypes.c_int
    L.ltxattn_comm_destroy.argtypes = [vp]
    L.ltxattn_comm_destroy.restype = ctypes.c_int
    L.ltxattn_allgather_heads.argtypes = [ctypes.POINTER(GatherArgs), vp, vp]
    L.ltxattn_allgather_heads.restype = ctypes.c_int
    L.ltxattn_device_count.argtypes = [ctypes.POINTER(ctypes.c_int32)]
    L.ltxattn_device_count.restype = ctypes.c_int
    L.ltxattn_device_query.argtypes = [ctypes.c_int32, ctypes.POINTER(DeviceInfo)]
    L.ltxattn_device_query.restype = ctypes.c_int
    L.ltxattn_last_error.argtypes = []
    L.ltxattn_last_error.restype = ctypes.c_char_p
    L.ltxattn_device_status.argtypes = [ctypes.c_int32, ctypes.POINTER(ctypes.c_int32)]
    L.ltxattn_device_status.restype = ctypes.c_int
    L.ltxattn_comm_size.argtypes = [vp, ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int32)]
    L.ltxattn_comm_size.restype = ctypes.c_int
    L.ltxattn_selftest_wait_timeout.argtypes = [ctypes.c_uint32, vp]
    L.ltxattn_selftest_wait_timeout.restype = ctypes.c_int
    L.ltxattn_memory_plan.argtypes = [ctypes.POINTER(MemoryPlanArgs), ctypes.POINTER(MemoryPlanInfo)]
    L.ltxattn_memory_plan.restype = ctypes.c_int
    L.ltxattn_linear.argtypes = [ctypes.POINTER(LinearArgs), vp]
    L.ltxattn_linear.restype = ctypes.c_int
    L.ltxattn_linear_workspace.argtypes = [ctypes.POINTER(LinearArgs)]
    L.ltxattn_linear_workspace.restype = ctypes.c_size_t
    L.ltxattn_head_gate.argtypes = [ctypes.POINTER(HeadGateArgs), vp]
    L.ltxattn_head_gate.restype = ctypes.c_int
    L.ltxattn_out_project_workspace.argtypes = [ctypes.POINTER(OutProjectArgs)]
    L.ltxattn_out_project_workspace.restype = ctypes.c_size_t
    L.ltxattn_out_project_allreduce.argtypes = [ctypes.POINTER(OutProjectArgs), vp, vp]
    L.ltxattn_out_project_allreduce.restype = ctypes.c_int
    L.ltxattn_abi_version.argtypes = []
    L.ltxattn_abi_version.restype = ctypes.c_int
    _lib = L
    return L


def last_error() -> str:
    return load().ltxattn_last_error().decode("utf-8", "replace")
