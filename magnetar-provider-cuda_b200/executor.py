"""``CudaExecutor``: the provider's ``ProviderExecutionApi`` surface for one device.

Mirrors ``impl ProviderExecutionApi for CudaExecutor`` (``src/executor.rs:2244-2565``):
tensors live in a device table keyed by resource id; ``submit_kernel`` runs an invocation
by kernel name with the reference's attribute rules and keeps the output resident; only
``read_tensor``/``read_tensor_rows`` bring data back to the host.  Everything runs in the
native library (``src/executor.rs:1422-2027`` is restated in ``csrc/executor.cu``).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Dict, Iterable, List, Mapping, Optional, Sequence, Union

import numpy as np

from . import _native as N
from ._native import CudaError, check
from .kernels import CudaKernels, DeviceBuffer

AttrValue = Union[bool, int, float, str]


@dataclass
class KernelInvocation:
    """One ``KernelInvocation``: kernel name, input ids, output id, attributes."""

    kernel: str
    inputs: Sequence[str]
    output: str
    attributes: Mapping[str, AttrValue] = field(default_factory=dict)
    input_dtypes: Optional[Sequence[str]] = None  # descriptor dtypes, e.g. ["f16", "f16"]
    deadline_millis: Optional[int] = None


@dataclass
class KernelResult:
    """``KernelResult``: success, or the failure's category and detail (kernel failures
    are reported inside the result, not raised, as ``src/executor.rs:1223-1231``)."""

    invocation_kernel: str
    output: str
    success: bool
    error_code: Optional[str] = None
    error_detail: Optional[str] = None


def _attributes(attrs: Mapping[str, AttrValue]):
    arr = (N.Attribute * max(1, len(attrs)))()
    keep = []
    for i, (name, value) in enumerate(attrs.items()):
        a = arr[i]
        bname = name.encode()
        keep.append(bname)
        a.name = bname
        if isinstance(value, bool):
            a.kind, a.int_value = N.ATTR_BOOL, int(value)
        elif isinstance(value, int):
            a.kind, a.int_value = N.ATTR_INT, value
        elif isinstance(value, float):
            a.kind, a.float_value = N.ATTR_FLOAT, value
        elif isinstance(value, str):
            s = value.encode()
            keep.append(s)
            a.kind, a.string_value = N.ATTR_STRING, s
        else:
            raise TypeError(f"attribute {name}: unsupported value {value!r}")
    return arr, keep


class CudaExecutor:
    """Executor of one device (``CudaExecutor``)."""

    def __init__(self, kernels: CudaKernels):
        self.kernels = kernels
        h = ctypes.c_void_p()
        check(N.lib().mg_executor_create(kernels.handle, ctypes.byref(h)))
        self._h = h
        self._comm = None

    @property
    def handle(self):
        return self._h

    def close(self) -> None:
        if self._h and self._h.value:
            N.lib().mg_executor_destroy(self._h)
            self._h = ctypes.c_void_p(0)

    # ---- tensors ------------------------------------------------------------------------
    def write_tensor(self, id: str, data, shape: Optional[Sequence[int]] = None) -> None:
        a = np.ascontiguousarray(data, dtype=np.float32)
        shape = tuple(a.shape) if shape is None else tuple(shape)
        check(N.lib().mg_executor_write_tensor(self._h, id.encode(), len(shape), N.shape_array(shape),
                                               a.ctypes.data))

    def write_weight_tensor(self, id: str, data, shape: Optional[Sequence[int]] = None) -> None:
        """A weight: under a tensor-parallel plan only this rank's share is kept."""
        a = np.ascontiguousarray(data, dtype=np.float32)
        shape = tuple(a.shape) if shape is None else tuple(shape)
        check(N.lib().mg_executor_write_weight_tensor(self._h, id.encode(), len(shape),
                                                      N.shape_array(shape), a.ctypes.data))

    def write_packed_weight_tensor(self, id: str, blocks, stored_rows: int, stored_cols: int,
                                   transposed: bool = True, format: str = "q8_0") -> None:
        """``write_packed_weight_tensor``: a Q8_0 weight kept as its 34-byte blocks' quants and scales."""
        if format != "q8_0":
            raise CudaError(2, f"packed weight format {format} is not supported")
        raw = np.ascontiguousarray(np.asarray(blocks, np.uint8).ravel())
        check(N.lib().mg_executor_write_packed_weight_tensor(self._h, id.encode(), N.PACKED_Q8_0, raw.ctypes.data,
                                                             raw.nbytes, stored_rows, stored_cols, 1 if transposed else 0))

    def write_zeroed_tensor(self, id: str, shape: Sequence[int]) -> None:
        check(N.lib().mg_executor_write_zeroed_tensor(self._h, id.encode(), len(shape), N.shape_array(shape)))

    def adopt(self, id: str, buf: DeviceBuffer) -> None:
        """Binds an existing device buffer as resource ``id`` (ownership moves here)."""
        check(N.lib().mg_executor_adopt_buffer(self._h, id.encode(), buf.handle))
        buf._h = ctypes.c_void_p(0)

    def buffer(self, id: str) -> DeviceBuffer:
        """A borrowed view of resource ``id`` (valid until it is rewritten)."""
        h = ctypes.c_void_p()
        check(N.lib().mg_executor_buffer(self._h, id.encode(), ctypes.byref(h)))
        return _BorrowedBuffer(h.value, self.kernels, self)

    def resident_shape(self, id: str) -> Optional[tuple]:
        present, rank = ctypes.c_int(), ctypes.c_int()
        dims = (ctypes.c_uint64 * N.MG_MAX_RANK)()
        check(N.lib().mg_executor_resident_shape(self._h, id.encode(), ctypes.byref(present),
                                                 ctypes.byref(rank), dims))
        return tuple(int(dims[i]) for i in range(rank.value)) if present.value else None

    def read_tensor(self, id: str) -> Optional[np.ndarray]:
        shape = self.resident_shape(id)
        if shape is None:
            return None
        out = np.empty(shape, dtype=np.float32)
        rank = ctypes.c_int()
        dims = (ctypes.c_uint64 * N.MG_MAX_RANK)()
        check(N.lib().mg_executor_read_tensor(self._h, id.encode(), out.ctypes.data, out.size,
                                              ctypes.byref(rank), dims))
        return out

    def read_tensor_rows(self, id: str, first_row: int, rows: int) -> Optional[np.ndarray]:
        shape = self.resident_shape(id)
        if shape is None or len(shape) != 2 or first_row + rows > shape[0]:
            return None
        out = np.empty((rows, shape[1]), dtype=np.float32)
        check(N.lib().mg_executor_read_tensor_rows(self._h, id.encode(), first_row, rows, out.ctypes.data,
                                                   out.size))
        return out

    def select_greedy_column(self, logits: str, row: int, excluded=(), temperature: float = 0.0) -> Optional[int]:
        """``select_greedy_column``: greedy selection over a resident logits tensor; None when
        no column is eligible or the selection fails (the reference's ``ok().flatten()``)."""
        found, column = ctypes.c_int(), ctypes.c_uint64()
        pairs, count = N.range_pairs(excluded)
        status = N.lib().mg_executor_select_greedy_column(self._h, logits.encode(), row, pairs, count,
                                                          ctypes.c_float(temperature), ctypes.byref(found),
                                                          ctypes.byref(column))
        return int(column.value) if status == 0 and found.value else None

    def release_tensor(self, id: str) -> bool:
        r = ctypes.c_int()
        check(N.lib().mg_executor_release_tensor(self._h, id.encode(), ctypes.byref(r)))
        return bool(r.value)

    def copy_tensor(self, src: str, dst: str) -> None:
        check(N.lib().mg_executor_copy_tensor(self._h, src.encode(), dst.encode()))

    # ---- kernels ------------------------------------------------------------------------
    def _invocation(self, inv: KernelInvocation):
        ids = [s.encode() for s in inv.inputs]
        inputs = (ctypes.c_char_p * max(1, len(ids)))(*ids)
        dtypes = None
        if inv.input_dtypes is not None:
            codes = [{"f32": N.F32, "f16": N.F16, "bf16": N.BF16}[d] for d in inv.input_dtypes]
            dtypes = (ctypes.c_int * max(1, len(codes)))(*codes)
        attrs, keep = _attributes(inv.attributes)
        c = N.Invocation()
        c.kernel = inv.kernel.encode()
        c.input_count = len(ids)
        c.inputs = ctypes.cast(inputs, ctypes.POINTER(ctypes.c_char_p))
        c.input_dtypes = ctypes.cast(dtypes, ctypes.POINTER(ctypes.c_int)) if dtypes is not None else None
        c.output = inv.output.encode()
        c.attribute_count = len(inv.attributes)
        c.attributes = ctypes.cast(attrs, ctypes.POINTER(N.Attribute))
        c.deadline_millis = -1 if inv.deadline_millis is None else int(inv.deadline_millis)
        return c, (ids, inputs, dtypes, attrs, keep)

    def run(self, inv: KernelInvocation) -> None:
        """Runs an invocation; raises ``CudaError`` on failure."""
        c, _keep = self._invocation(inv)
        check(N.lib().mg_executor_submit_kernel(self._h, ctypes.byref(c)))

    def submit_kernel(self, inv: KernelInvocation) -> KernelResult:
        """``submit_kernel`` + ``complete_kernel``: failures come back inside the result."""
        try:
            self.run(inv)
            return KernelResult(inv.kernel, inv.output, True)
        except CudaError as e:
            return KernelResult(inv.kernel, inv.output, False, e.code, e.detail)

    def synchronize(self) -> None:
        check(N.lib().mg_executor_synchronize(self._h))

    # ---- step capture ---------------------------------------------------------------------
    def begin_step_capture(self, advancing: Sequence[str] = ()) -> None:
        """Records the following invocations into one replayable step.  ``advancing`` names
        the attributes a replay's offset is added to ("position_offset", "key_count",
        "row_offset"; the reference's StepCaptureRequest advancing_attributes)."""
        if not advancing:
            check(N.lib().mg_executor_begin_step_capture(self._h))
            return
        names = (ctypes.c_char_p * len(advancing))(*[a.encode() for a in advancing])
        check(N.lib().mg_executor_begin_step_capture_advancing(self._h, names, len(advancing)))

    def end_step_capture(self) -> None:
        check(N.lib().mg_executor_end_step_capture(self._h))

    def abort_step_capture(self) -> None:
        check(N.lib().mg_executor_abort_step_capture(self._h))

    def replay_step(self, offset: int = 0) -> None:
        """One replay (with the embedding-id check) at ``offset`` for the advancing attributes."""
        if offset:
            check(N.lib().mg_executor_replay_step_at(self._h, int(offset)))
        else:
            check(N.lib().mg_executor_replay_step(self._h))

    def replay_step_io(self, inputs: Mapping[str, object] = None, outputs: Mapping[str, object] = None,
                       offset: int = 0) -> None:
        """One replay with its host I/O in one call (``replay_step(id, offset, inputs)`` plus the
        step's reads): ``inputs`` / ``outputs`` map ids to contiguous host arrays (numpy arrays or
        pinned torch tensors) of exactly the buffers' bytes; one synchronisation covers the
        copies and the embedding-id check."""
        self.step_io(inputs, outputs)(offset)

    def step_io(self, inputs: Mapping[str, object] = None, outputs: Mapping[str, object] = None):
        """The host I/O of ``replay_step_io`` described once: returns ``replay(offset=0)``, which
        replays with those arrays (their contents may change between calls, not their storage)."""
        return self._step_io(N.lib().mg_executor_replay_step_io, (self._h,), inputs, outputs)

    # ---- several captured steps (StepCaptureId) ----------------------------------------------
    def end_step_capture_id(self) -> int:
        """``end_step_capture``: ends the capture, keeps the step under a new id and runs it once
        (its results are then available), as ``src/executor.rs`` end_step_capture does."""
        v = ctypes.c_uint64()
        check(N.lib().mg_executor_end_step_capture_id(self._h, ctypes.byref(v)))
        return v.value

    def replay_capture(self, step_id: int, offset: int = 0, inputs: Mapping[str, object] = None,
                       outputs: Mapping[str, object] = None) -> None:
        """``replay_step(id, offset, inputs)``, with ``outputs`` read back in the same call."""
        self.capture_io(step_id, inputs, outputs)(offset)

    def capture_io(self, step_id: int, inputs: Mapping[str, object] = None, outputs: Mapping[str, object] = None):
        """``replay_capture``'s host I/O described once: returns ``replay(offset=0)``."""
        return self._step_io(N.lib().mg_executor_replay_capture, (self._h, int(step_id)), inputs, outputs)

    def release_step_capture(self, step_id: int) -> None:
        check(N.lib().mg_executor_release_step_capture(self._h, int(step_id)))

    def step_capture_count(self) -> int:
        v = ctypes.c_int()
        check(N.lib().mg_executor_step_capture_count(self._h, ctypes.byref(v)))
        return v.value

    def _step_io(self, fn, lead, inputs, outputs):
        entries = []
        keep = []
        for mapping, to_dev in ((inputs or {}, 1), (outputs or {}, 0)):
            for id, arr in mapping.items():
                if hasattr(arr, "data_ptr"):  # a torch tensor
                    ptr, nbytes = arr.data_ptr(), arr.numel() * arr.element_size()
                else:
                    a = np.asarray(arr)
                    if not a.flags["C_CONTIGUOUS"] or (not to_dev and not a.flags["WRITEABLE"]):
                        raise ValueError(f"{id}: host arrays must be contiguous (and writable for outputs)")
                    ptr, nbytes = a.ctypes.data, a.nbytes
                    keep.append(a)
                key = id.encode()
                keep.append(key)
                entries.append(N.StepIO(key, ptr, nbytes, to_dev))
        arr_t = (N.StepIO * max(1, len(entries)))(*entries)
        ptr, count = ctypes.cast(arr_t, ctypes.c_void_p), len(entries)
        refs = (arr_t, keep, inputs, outputs)  # kept alive with the closure

        def replay(offset: int = 0) -> None:
            check(fn(*lead, offset, ptr, count))

        replay.refs = refs
        return replay

    def step_max_offset(self) -> int:
        """The largest offset the captured step accepts (2**64 - 1: unbounded)."""
        v = ctypes.c_uint64()
        check(N.lib().mg_executor_step_max_offset(self._h, ctypes.byref(v)))
        return v.value

    def replay_steps(self, count: int) -> None:
        """``count`` replays back to back with one embedding-id check for all of them."""
        if count < 1:
            raise ValueError("count must be positive")
        check(N.lib().mg_executor_replay_steps(self._h, int(count)))

    def launch_step(self) -> None:
        """One replay without the embedding-id check (``check_steps`` checks later)."""
        check(N.lib().mg_executor_launch_step(self._h))

    def check_steps(self) -> None:
        """Checks the embedding ids of every replay since the last check."""
        check(N.lib().mg_executor_check_steps(self._h))

    def observations(self) -> Dict[str, int]:
        s, c, f = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
        check(N.lib().mg_executor_observations(self._h, ctypes.byref(s), ctypes.byref(c), ctypes.byref(f)))
        return {"started": s.value, "completed": c.value, "failed": f.value}

    def observation_log(self) -> List[Dict[str, object]]:
        """The most recent ``KernelObservation`` events, oldest first (at most 4096):
        ``{"kind", "kernel", "invocation", "error"}`` (``error`` the failure's status name)."""
        n = ctypes.c_uint32()
        check(N.lib().mg_executor_observation_log(self._h, None, 0, ctypes.byref(n)))
        arr = (N.Observation * max(1, n.value))()
        check(N.lib().mg_executor_observation_log(self._h, ctypes.cast(arr, ctypes.c_void_p), n.value, ctypes.byref(n)))
        return [{"kind": N.OBSERVATION_KINDS.get(o.kind, str(o.kind)), "kernel": o.kernel.decode(),
                 "invocation": o.invocation, "error": N.STATUS_NAMES.get(o.status) if o.status else None}
                for o in arr[:n.value]]

    # ---- tensor parallel -------------------------------------------------------------------
    def attach_comm(self, comm) -> None:
        self._comm = comm
        check(N.lib().mg_executor_attach_comm(self._h, comm.handle if comm is not None else None))

    def apply_tensor_parallel(self, plan: Mapping[str, str]) -> None:
        """``apply_tensor_parallel``: weight id -> "columns" | "rows"."""
        ids = [k.encode() for k in plan]
        kinds = [{"columns": 0, "rows": 1}[v] for v in plan.values()]
        arr = (ctypes.c_char_p * max(1, len(ids)))(*ids)
        karr = (ctypes.c_int * max(1, len(kinds)))(*kinds)
        check(N.lib().mg_executor_apply_tensor_parallel(self._h, len(ids), arr, karr))


class _BorrowedBuffer(DeviceBuffer):
    """A view of an executor-owned buffer; releasing it does nothing."""

    __slots__ = ()

    def release(self) -> None:
        self._h = ctypes.c_void_p(0)
