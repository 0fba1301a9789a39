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

import numpy as np
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


class _IpcBlock:
    """One cudaMalloc block per rank (zeroed), mapped on every rank's device: the
    blocks' CUDA IPC handles are exchanged through ``torch.distributed`` and opened
    with lazy peer access, so ``peer_base[d]`` is rank d's block on this device
    (``peer_base[rank]`` the own one).  Collective: every rank builds and closes
    its block together."""

    def __init__(self, nbytes: int, group=None):
        from cuda.bindings import runtime as cudart
        self._rt = cudart
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 2 <= self.world <= 8:
            raise Failure("arg", f"world {self.world}: peer-memory collectives join 2 to 8 ranks", _lib.ERR_ARG)
        self.device = torch.cuda.current_device()
        self._ok(cudart.cudaSetDevice(self.device))
        self.base = int(self._ok(cudart.cudaMalloc(nbytes)))
        self._ok(cudart.cudaMemset(self.base, 0, nbytes))
        self._ok(cudart.cudaDeviceSynchronize())
        mine = bytes(self._ok(cudart.cudaIpcGetMemHandle(self.base)).reserved)
        handles = [None] * self.world
        dist.all_gather_object(handles, mine, group=group)
        self._opened = []
        self.peer_base = []
        for d, h in enumerate(handles):
            if d == self.rank:
                self.peer_base.append(self.base)
                continue
            ph = cudart.cudaIpcMemHandle_t()
            ph.reserved = h
            ptr = int(self._ok(cudart.cudaIpcOpenMemHandle(ph, cudart.cudaIpcMemLazyEnablePeerAccess)))
            self._opened.append(ptr)
            self.peer_base.append(ptr)
        dist.barrier(group=group)  # every rank has mapped every block before any call stores into it

    @staticmethod
    def _ok(res):
        err = res[0]
        if int(err) != 0:
            raise Failure("cuda", f"CUDA runtime call failed: {err}", _lib.ERR_CUDA)
        return res[1] if len(res) > 1 else None

    def tensor(self, offset: int, shape, dtype):
        """A torch view of this rank's block at byte `offset` (bf16 / int32 / float32)."""
        elems = {torch.bfloat16: 1, torch.int32: 2, torch.float32: 2}[dtype]
        n16 = int(np.prod(shape)) * elems
        t = torch.as_tensor(_DeviceArray(self.base + offset, (n16,)), device=torch.device("cuda", self.device))
        return t.view(dtype).view(tuple(shape))

    def close(self):
        torch.cuda.synchronize()
        dist.barrier(group=self.group)  # no rank still stores into a block about to be unmapped
        for ptr in self._opened:
            self._ok(self._rt.cudaIpcCloseMemHandle(ptr))
        self._opened = []
        dist.barrier(group=self.group)
        if self.base:
            self._ok(self._rt.cudaFree(self.base))
            self.base = 0


_SIG_BYTES = 256  # 16 uint32 signal words, padded so what follows is 256-byte aligned


class FusedHeadGather:
    """Buffers and calls of ``ltxattn_fwd_gather``: the head-sharded attention
    whose epilogue stores each output tile into every rank's output over NVLink
    (the all-gather fused into the attention).

    Each rank's IPC block (``_IpcBlock``) holds 16 signal words, then its full
    output ``out`` [B, H, T, D] bf16.  ``run`` computes this rank's head block
    (``head_block``) and returns with every rank's heads in ``out`` (stream
    ordered).  Every rank must call ``run`` the same number of times with the
    same shapes; ``close`` releases the mappings (collective)."""

    def __init__(self, shape, group=None):
        B, H, T, D = (int(x) for x in shape)
        self.shape = (B, H, T, D)
        self.block = _IpcBlock(_SIG_BYTES + B * H * T * D * 2, group)
        self.world, self.rank = self.block.world, self.block.rank
        self.out = self.block.tensor(_SIG_BYTES, (B, H, T, D), torch.bfloat16)
        self.epoch = 0
        self._peers = _lib.GatherPeers()
        self._peers.world, self._peers.rank = self.world, self.rank
        for d, b in enumerate(self.block.peer_base):
            self._peers.out[d] = b + _SIG_BYTES
            self._peers.signals[d] = b

    def run(self, q, k, v, scale: Optional[float] = None, q_rotary=None, k_rotary=None, stream=None):
        """This rank's head block of attention(q, k, v) (full [B, H, T, D] inputs on
        this device; only the block's heads are read), gathered into ``out`` on
        every rank."""
        from .backend import AttentionBackend, _stream_ptr
        H, D = self.shape[1], self.shape[3]
        h0, hc = head_block(H, self.world, self.rank)
        if scale is None:
            scale = 1.0 / float(D) ** 0.5
        a, _ = AttentionBackend.make_fwd_args(q, k, v, scale, q_rotary=q_rotary, k_rotary=k_rotary, out=self.out,
                                              head_begin=h0, head_count=hc)
        L = _lib.load()
        n = int(L.ltxattn_fwd_workspace(ctypes.byref(a)))
        ws = None
        if n > 0:
            ws = torch.empty(n + 256, dtype=torch.uint8, device=q.device)
            a.workspace = (ws.data_ptr() + 255) // 256 * 256
            a.workspace_bytes = n
        self.epoch += 1
        self._peers.epoch = self.epoch
        rc = L.ltxattn_fwd_gather(ctypes.byref(a), ctypes.byref(self._peers), ctypes.c_void_p(_stream_ptr(stream)))
        if rc != _lib.OK:
            raise Failure.from_status(rc)
        self._ws = ws  # the workspace lives until the next call (stream-ordered use)
        return self.out

    def close(self):
        self.block.close()


class FusedOutProject:
    """Buffers and calls of ``ltxattn_out_project_fused``: the row-parallel to_out
    whose reduction runs over peer memory (the GEMM's epilogue stores each fp32
    partial row into its owner's receive plane, owners add the planes in rank order
    and store the rounded rows into every rank's output).

    Each rank's IPC block holds 16 signal words, ``world`` fp32 receive planes of
    [m, n], then its output ``out`` [m, n] bf16.  Collective like
    ``FusedHeadGather``."""

    def __init__(self, m: int, n: int, group=None):
        self.m, self.n = int(m), int(n)
        world = dist.get_world_size(group)
        recv_bytes = world * self.m * self.n * 4
        self._off_out = _SIG_BYTES + (recv_bytes + 255) // 256 * 256
        self.block = _IpcBlock(self._off_out + self.m * self.n * 2, group)
        self.world, self.rank = self.block.world, self.block.rank
        self.out = self.block.tensor(self._off_out, (self.m, self.n), torch.bfloat16)
        self.epoch = 0
        self._peers = _lib.ReducePeers()
        self._peers.world, self._peers.rank = self.world, self.rank
        for d, b in enumerate(self.block.peer_base):
            self._peers.recv[d] = b + _SIG_BYTES
            self._peers.out[d] = b + self._off_out
            self._peers.signals[d] = b

    def run(self, x_local: torch.Tensor, weight_block: torch.Tensor, bias: Optional[torch.Tensor] = None,
            stream=None) -> torch.Tensor:
        """to_out of this rank's merged head slice x_local [m, k] with its column block
        of to_out.0.weight [n, k]; returns ``out`` [m, n] holding the whole sum on every
        rank (stream ordered)."""
        from .backend import _stream_ptr
        k = x_local.shape[-1]
        x2 = x_local.reshape(-1, k)
        if x2.shape[0] != self.m or weight_block.shape[0] != self.n or weight_block.shape[1] != k or \
                weight_block.stride(1) != 1:
            raise Failure.shape("x_local / weight_block", tuple(x2.shape) + tuple(weight_block.shape),
                                f"[{self.m}, k] and [{self.n}, k]")
        a = _lib.OutProjectArgs()
        a.dtype, a.m, a.n, a.k = _lib.BF16, self.m, self.n, k
        a.x, a.x_stride = x2.data_ptr(), x2.stride(0) if self.m > 1 else k
        a.weight, a.weight_stride = weight_block.data_ptr(), weight_block.stride(0)
        a.bias = bias.data_ptr() if bias is not None else None
        a.out, a.out_stride = self.out.data_ptr(), self.n
        self.epoch += 1
        self._peers.epoch = self.epoch
        rc = _lib.load().ltxattn_out_project_fused(ctypes.byref(a), ctypes.byref(self._peers),
                                                   ctypes.c_void_p(_stream_ptr(stream)))
        if rc != _lib.OK:
            raise Failure.from_status(rc)
        return self.out

    def close(self):
        self.block.close()


class _DeviceArray:
    """A device pointer with a shape, for torch.as_tensor (int16 elements)."""

    def __init__(self, ptr: int, shape):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": tuple(shape), "typestr": "<i2",
                                         "version": 3, "strides": None}
