"""Head-parallel plumbing: which heads a rank owns, the NCCL id exchange, the
head all-gather, and the max-over-ranks timing reduction.

The reference runs one job on one device (``Sources/LTX25/RenderEngine.swift:16-24``);
attention heads are independent, so a job spread over the GPUs of one box
gives each rank a contiguous block of heads and needs no communication inside
attention.  ``HeadGather`` wraps ``ltxattn_allgather_heads`` (NCCL over
NVLink) for callers that need every head on every rank.

``torch.distributed`` carries the 128-byte NCCL id and the timing reduction;
any backend works for those (the CPU tests use gloo).
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib
from .backend import Failure


def head_block(heads: int, world: int, rank: int) -> Tuple[int, int]:
    """(head_begin, head_count) of ``rank``: contiguous, equal blocks."""
    if world < 1 or not 0 <= rank < world:
        raise Failure("arg", f"rank {rank} of world {world}", _lib.ERR_ARG)
    if heads % world:
        raise Failure.shape("heads", [heads], f"a multiple of the {world} ranks")
    per = heads // world
    return rank * per, per


def exchange_unique_id(group=None, make_id=None) -> bytes:
    """Rank 0 creates the 128-byte NCCL id; every rank returns the same bytes."""
    rank = dist.get_rank(group)
    buf = torch.zeros(128, dtype=torch.uint8)
    if rank == 0:
        if make_id is None:
            raw = (ctypes.c_uint8 * 128)()
            rc = _lib.load().ltxattn_comm_unique_id(raw)
            if rc != _lib.OK:
                raise Failure.from_status(rc)
            make_id = bytes(raw)
        elif callable(make_id):
            make_id = make_id()
        buf.copy_(torch.frombuffer(bytearray(make_id), dtype=torch.uint8))
    if dist.get_backend(group) == "nccl":
        dev = torch.device("cuda", torch.cuda.current_device())
        b = buf.to(dev)
        dist.broadcast(b, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
        buf = b.cpu()
    else:
        dist.broadcast(buf, src=0, group=group)
    return bytes(buf.tolist())


def max_over_ranks(values, group=None):
    """Element-wise max of a list of floats over all ranks (device times)."""
    t = torch.tensor(list(values), dtype=torch.float64)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        if dist.get_backend(group) == "nccl":
            t = t.cuda()
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return t.cpu().tolist()


class HeadGather:
    """NCCL communicator owned by libltxattn_cuda, for ``ltxattn_allgather_heads``."""

    def __init__(self, world: int, rank: int, unique_id: bytes, device: int):
        L = _lib.load()
        self._comm = ctypes.c_void_p()
        raw = (ctypes.c_uint8 * 128).from_buffer_copy(unique_id)
        rc = L.ltxattn_comm_init(ctypes.byref(self._comm), world, rank, raw, device)
        if rc != _lib.OK:
            raise Failure.from_status(rc)
        self.world, self.rank = world, rank

    def size(self) -> Tuple[int, int]:
        """(ranks, this rank) as NCCL reports them for the communicator."""
        n, r = ctypes.c_int32(), ctypes.c_int32()
        rc = _lib.load().ltxattn_comm_size(self._comm, ctypes.byref(n), ctypes.byref(r))
        if rc != _lib.OK:
            raise Failure.from_status(rc)
        return n.value, r.value

    def gather(self, local: torch.Tensor, out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
        """[B, H/N, T, D] contiguous on every rank -> [B, H, T, D] on every rank."""
        if not local.is_contiguous() or local.dim() != 4:
            raise Failure.shape("local", local.shape, "a contiguous [B, heads_per_rank, T, D]")
        B, hpr, T, D = local.shape
        if out is None:
            out = torch.empty((B, hpr * self.world, T, D), dtype=local.dtype, device=local.device)
        a = _lib.GatherArgs()
        a.dtype = _lib.BF16 if local.dtype == torch.bfloat16 else _lib.F32
        a.batch, a.heads_per_rank, a.tokens, a.head_dim = B, hpr, T, D
        a.send, a.recv = local.data_ptr(), out.data_ptr()
        s = stream if stream is not None else torch.cuda.current_stream()
        rc = _lib.load().ltxattn_allgather_heads(ctypes.byref(a), self._comm, ctypes.c_void_p(s.cuda_stream))
        if rc != _lib.OK:
            raise Failure.from_status(rc)
        return out

    def out_project(self, x_local: torch.Tensor, weight_block: torch.Tensor, bias: Optional[torch.Tensor] = None,
                    out: Optional[torch.Tensor] = None, workspace: Optional[torch.Tensor] = None,
                    stream=None) -> torch.Tensor:
        """Row-parallel to_out (``ltxattn_out_project_allreduce``): this rank's merged
        head slice x_local [..., k] times its column block of to_out.0.weight
        ([n, k], any row stride), summed over the ranks, + bias; every rank gets
        [..., n]."""
        k = x_local.shape[-1]
        x2 = x_local.reshape(-1, k)
        m, n = x2.shape[0], weight_block.shape[0]
        if weight_block.dim() != 2 or weight_block.shape[1] != k or weight_block.stride(1) != 1:
            raise Failure.shape("weight_block", weight_block.shape, f"[n, {k}] with unit stride along k")
        if out is None:
            out = torch.empty(x_local.shape[:-1] + (n,), dtype=x_local.dtype, device=x_local.device)
        a = _lib.OutProjectArgs()
        a.dtype, a.m, a.n, a.k = _lib.BF16, m, n, k
        a.x, a.x_stride = x2.data_ptr(), x2.stride(0) if m > 1 else k
        a.weight, a.weight_stride = weight_block.data_ptr(), weight_block.stride(0)
        a.bias = bias.data_ptr() if bias is not None else None
        o2 = out.view(-1, n)
        a.out, a.out_stride = o2.data_ptr(), o2.stride(0) if m > 1 else n
        L = _lib.load()
        need = int(L.ltxattn_out_project_workspace(ctypes.byref(a)))
        if workspace is None or workspace.numel() * workspace.element_size() < need:
            workspace = torch.empty(need, dtype=torch.uint8, device=x_local.device)
        a.workspace, a.workspace_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
        s = stream if stream is not None else torch.cuda.current_stream()
        rc = L.ltxattn_out_project_allreduce(ctypes.byref(a), self._comm, ctypes.c_void_p(s.cuda_stream))
        if rc != _lib.OK:
            raise Failure.from_status(rc)
        return out

    def close(self):
        if self._comm:
            _lib.load().ltxattn_comm_destroy(self._comm)
            self._comm = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def gather_layout(blocks):
    """The layout contract of ltxattn_allgather_heads, for host-side checks: rank r's
    [B, H/N, T, D] block lands at heads [r*H/N, (r+1)*H/N) of [B, H, T, D]."""
    return torch.cat(list(blocks), dim=1)
