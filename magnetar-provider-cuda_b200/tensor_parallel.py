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


class PeerLost(RuntimeError):
    """A rank of the group did not reach a step in time (it exited, hung or was killed)."""

    def __init__(self, step: int, missing):
        self.step, self.missing = step, sorted(missing)
        super().__init__(f"rank(s) {self.missing} did not reach step {step} in time")


class StepMonitor:
    """Host-side liveness of a group's ranks between steps, over a ``torch.distributed`` store.

    Before each step every rank posts its arrival and waits, bounded, for every peer's; a rank
    that exited or hung between steps is noticed there, on the host, before any kernel or
    collective of the next step is enqueued -- so nothing waits on it on the device.  The
    reference drives its members from one host thread and has no such failure path."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 30.0, prefix: str = "mg-step"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.prefix = float(timeout_s), prefix

    def _key(self, step: int, rank: int) -> str:
        return f"{self.prefix}/{step}/{rank}"

    def arrive(self, step: int) -> None:
        self.store.set(self._key(step, self.rank), "1")

    def check_peers(self, step: int) -> None:
        """Raises ``PeerLost`` naming the ranks that have not arrived at ``step`` within the
        timeout."""
        import datetime
        keys = [self._key(step, r) for r in range(self.world)]
        try:
            self.store.wait(keys, datetime.timedelta(seconds=self.timeout_s))
        except Exception:
            missing = [r for r, k in enumerate(keys) if not self.store.check([k])]
            raise PeerLost(step, missing or list(range(self.world))) from None

    def step(self, step: int) -> None:
        self.arrive(step)
        self.check_peers(step)


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

    # ---- failure handling: every NCCL call is bounded by the group's timeout -------------------
    def set_timeout(self, timeout_ms: int) -> None:
        """Host time after which a pending NCCL call aborts the communicator."""
        check(N.lib().mg_comm_set_timeout(self._h, int(timeout_ms)))

    def check(self) -> None:
        """Raises (and aborts the communicator) if NCCL reported an asynchronous error."""
        check(N.lib().mg_comm_check(self._h))

    def wait(self, timeout_ms: int = 0) -> None:
        """Waits for this rank's enqueued group work; aborts after ``timeout_ms`` (0: the
        group's timeout) and raises ``DeviceUnavailable``."""
        check(N.lib().mg_comm_wait(self._h, int(timeout_ms)))

    def abort(self) -> None:
        """Aborts the communicator at once (a peer is known to be gone)."""
        check(N.lib().mg_comm_abort(self._h))

    @property
    def aborted(self) -> bool:
        return bool(N.lib().mg_comm_is_aborted(self._h))

    def begin_step(self, monitor: "StepMonitor", step: int) -> None:
        """Checks on the host that every rank reached ``step`` before its work is enqueued; a
        lost peer aborts the communicator and raises ``PeerLost``."""
        try:
            monitor.step(step)
        except PeerLost:
            self.abort()
            raise

    def mlp(self, x: DeviceBuffer, gate_shard: DeviceBuffer, up_shard: DeviceBuffer, down_shard: DeviceBuffer,
            chunks: int = 4, out: DeviceBuffer = None) -> DeviceBuffer:
        """y = sum over ranks of (silu(x G_r) * (x U_r)) D_r."""
        o = ctypes.c_void_p(out.handle.value if out is not None else None)
        check(N.lib().mg_tp_mlp(self._h, x.handle, gate_shard.handle, up_shard.handle, down_shard.handle,
                                int(chunks), ctypes.byref(o)))
        if out is not None and o.value == out.handle.value:
            return out
        return DeviceBuffer(o.value, self.kernels)

    def set_mlp_timing(self, on: bool = True) -> None:
        """Record events around each ``mlp`` call (see ``mlp_timing``)."""
        check(N.lib().mg_comm_set_mlp_timing(self._h, int(bool(on))))

    def mlp_timing(self):
        """(compute_ms, exposed_allreduce_ms) of the last timed ``mlp`` call: start to the end of
        its last down-projection chunk, and from there to the all-reduce stream's join."""
        c, e = ctypes.c_float(), ctypes.c_float()
        check(N.lib().mg_comm_mlp_timing(self._h, ctypes.byref(c), ctypes.byref(e)))
        return float(c.value), float(e.value)

    def close(self) -> None:
        if self._h and self._h.value:
            N.lib().mg_comm_destroy(self._h)
            self._h = ctypes.c_void_p(0)
