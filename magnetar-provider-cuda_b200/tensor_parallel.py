"""Tensor-parallel SwiGLU MLP across the GPUs of one box, one process per GPU.

Mirrors ``src/multi/tensor_parallel.rs``: gate/up weights split by columns, down by rows
(``WeightShard::{Columns, Rows}``), shares aligned to 32-element blocks when every part can
hold one (``share_granule``, ``:300-307``), and the partial outputs of a row-split
projection summed across members (``all_reduce``, ``:697-734``).  The reference drives all
members from one thread and sums serially through a root GPU; here each rank is its own
process, joins one NCCL communicator (the 128-byte id travels over ``torch.distributed``),
and the sum is one all-reduce overlapped with the down projection in row chunks.
"""
from __future__ import annotations

import ctypes
from typing import Tuple

import numpy as np

from . import _native as N
from ._native import check
from .kernels import CudaKernels, DeviceBuffer


def share_granule(extent: int, parts: int) -> int:
    """32 (a Q8_0 block) when ``extent`` splits into whole blocks for every part, else 1."""
    return 32 if extent % 32 == 0 and extent >= 32 * parts else 1


def share(extent: int, parts: int, member: int) -> Tuple[int, int]:
    """The ``[start, end)`` share of ``extent`` that ``member`` of ``parts`` holds."""
    if parts <= 0 or not 0 <= member < parts:
        raise ValueError(f"member {member} of {parts} parts")
    g = share_granule(extent, parts)
    units = extent // g
    return units * member // parts * g, units * (member + 1) // parts * g


def native_share(extent: int, parts: int, member: int) -> Tuple[int, int]:
    """``share`` computed by the native library (the executor's own rule)."""
    s, e = ctypes.c_uint64(), ctypes.c_uint64()
    check(N.lib().mg_tp_share(extent, parts, member, ctypes.byref(s), ctypes.byref(e)))
    return s.value, e.value


def split_columns(weight: np.ndarray, parts: int, member: int) -> np.ndarray:
    """``WeightShard::Columns``: this member's share of the last dimension."""
    s, e = share(weight.shape[-1], parts, member)
    return np.ascontiguousarray(weight[..., s:e])


def split_rows(weight: np.ndarray, parts: int, member: int) -> np.ndarray:
    """``WeightShard::Rows``: this member's share of the first dimension."""
    s, e = share(weight.shape[0], parts, member)
    return np.ascontiguousarray(weight[s:e])


class TpGroup:
    """This process's rank of a tensor-parallel group (an NCCL communicator)."""

    def __init__(self, kernels: CudaKernels, rank: int, world: int, unique_id: bytes):
        if len(unique_id) != 128:
            raise ValueError("a communicator id is 128 bytes")
        self.kernels = kernels
        self.rank, self.world = rank, world
        h = ctypes.c_void_p()
        check(N.lib().mg_comm_init(kernels.handle, rank, world, unique_id, ctypes.byref(h)))
        self._h = h

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(128)
        check(N.lib().mg_comm_unique_id(buf))
        return buf.raw

    @classmethod
    def from_torch_distributed(cls, kernels: CudaKernels) -> "TpGroup":
        """Joins the group of the initialised ``torch.distributed`` world (rank 0 makes the
        id, every rank receives it by broadcast)."""
        import torch
        import torch.distributed as dist
        rank, world = dist.get_rank(), dist.get_world_size()
        backend = dist.get_backend()
        dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
        t = torch.zeros(128, dtype=torch.uint8, device=dev)
        if rank == 0:
            t.copy_(torch.frombuffer(bytearray(cls.unique_id()), dtype=torch.uint8))
        dist.broadcast(t, 0)
        return cls(kernels, rank, world, bytes(t.cpu().numpy().tobytes()))

    @property
    def handle(self):
        return self._h

    def all_reduce(self, buf: DeviceBuffer) -> None:
        check(N.lib().mg_comm_all_reduce(self._h, buf.handle))

    def mlp(self, x: DeviceBuffer, gate_shard: DeviceBuffer, up_shard: DeviceBuffer, down_shard: DeviceBuffer,
            chunks: int = 4, out: DeviceBuffer = None) -> DeviceBuffer:
        """y = sum over ranks of (silu(x G_r) * (x U_r)) D_r."""
        o = ctypes.c_void_p(out.handle.value if out is not None else None)
        check(N.lib().mg_tp_mlp(self._h, x.handle, gate_shard.handle, up_shard.handle, down_shard.handle,
                                int(chunks), ctypes.byref(o)))
        if out is not None and o.value == out.handle.value:
            return out
        return DeviceBuffer(o.value, self.kernels)

    def close(self) -> None:
        if self._h and self._h.value:
            N.lib().mg_comm_destroy(self._h)
            self._h = ctypes.c_void_p(0)
