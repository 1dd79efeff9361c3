"""Device-level API: ``CudaKernels`` and ``DeviceBuffer``.

Mirrors the reference's ``CudaKernels`` launch wrappers (``src/kernels.rs:538-7132``) --
same operator names, argument meaning and error categories -- over the C ABI of
``libmagnetar_cuda.so``.  Buffers are device-resident; only ``upload``/``download`` and the
data-dependent checks (embedding ids, softmax rows) cross to the host.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence

import numpy as np

from . import _native as N
from ._native import CudaError, check

_DTYPES = {"f32": N.F32, "f16": N.F16, "bf16": N.BF16, "q8_0": N.Q8_0}
_DTYPE_NAMES = {v: k for k, v in _DTYPES.items()}


def _dtype_code(dtype) -> int:
    if isinstance(dtype, int):
        return dtype
    return _DTYPES[str(dtype)]


class DeviceBuffer:
    """A device tensor (``CudaDeviceBuffer`` / ``CudaHalfBuffer``): dtype, shape, memory."""

    __slots__ = ("_h", "_kernels", "_owner")

    def __init__(self, handle: int, kernels: "CudaKernels", owner=None):
        self._h = ctypes.c_void_p(handle)
        self._kernels = kernels
        self._owner = owner  # keeps a wrapped framework tensor alive

    @property
    def handle(self):
        return self._h

    @property
    def shape(self) -> tuple:
        rank = ctypes.c_int()
        dims = (ctypes.c_uint64 * N.MG_MAX_RANK)()
        check(N.lib().mg_buffer_shape(self._h, ctypes.byref(rank), dims))
        return tuple(int(dims[i]) for i in range(rank.value))

    @property
    def dtype(self) -> str:
        d = ctypes.c_int()
        check(N.lib().mg_buffer_dtype(self._h, ctypes.byref(d)))
        return _DTYPE_NAMES[d.value]

    @property
    def size(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n

    def data_ptr(self) -> int:
        return int(N.lib().mg_buffer_device_ptr(self._h) or 0)

    def reshape(self, shape: Sequence[int]) -> "DeviceBuffer":
        check(N.lib().mg_buffer_reshape(self._h, len(shape), N.shape_array(shape)))
        return self

    def set_weight(self, is_weight: bool = True) -> "DeviceBuffer":
        """Marks the buffer as a weight (``write_weight_tensor``): a matmul that reads it as B
        keeps B's tensor-core operand form with it instead of re-deriving it per call."""
        check(N.lib().mg_buffer_set_weight(self._h, 1 if is_weight else 0))
        return self

    def write(self, array) -> "DeviceBuffer":
        """Overwrites the buffer with host f32 values of the same element count (a weight
        drops its prepared and compact forms)."""
        a = np.ascontiguousarray(array, dtype=np.float32)
        check(N.lib().mg_buffer_upload_f32(self._h, a.ctypes.data, a.size))
        return self

    def is_q8(self) -> bool:
        """Whether this is a packed Q8_0 weight (``CudaDeviceBuffer::is_q8``)."""
        return bool(N.lib().mg_buffer_is_q8(self._h))

    def is_compact(self) -> bool:
        """Whether this weight holds its compact (bfloat16-bit) form, which the few-row matmul
        streams in place of the f32 values (``CudaDeviceBuffer::is_compact``)."""
        return bool(N.lib().mg_buffer_is_compact(self._h))

    def release(self) -> None:
        if self._h and self._h.value:
            N.lib().mg_buffer_release(self._h)
            self._h = ctypes.c_void_p(0)

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass

    def __repr__(self):
        return f"DeviceBuffer({self.dtype}, {self.shape})"


class CudaKernels:
    """Kernels of one device (``CudaKernels``, ``src/kernels.rs:538-616``)."""

    def __init__(self, ordinal: int = 0):
        h = ctypes.c_void_p()
        check(N.lib().mg_device_open(int(ordinal), ctypes.byref(h)))
        self._h = h
        self.ordinal = int(ordinal)

    @property
    def handle(self):
        return self._h

    def close(self) -> None:
        if self._h and self._h.value:
            N.lib().mg_device_close(self._h)
            self._h = ctypes.c_void_p(0)

    def info(self) -> dict:
        i = N.DeviceInfo()
        check(N.lib().mg_device_get_info(self._h, ctypes.byref(i)))
        return {"ordinal": i.ordinal, "name": i.name.decode(), "sm": f"sm_{i.sm_major}{i.sm_minor}",
                "sm_count": i.sm_count, "total_bytes": i.total_bytes, "free_bytes": i.free_bytes}

    def synchronize(self) -> None:
        check(N.lib().mg_device_synchronize(self._h))

    @property
    def stream(self) -> int:
        return int(N.lib().mg_device_stream(self._h) or 0)

    def set_stream(self, stream: Optional[int]) -> None:
        check(N.lib().mg_device_set_stream(self._h, ctypes.c_void_p(stream or 0)))

    def upload_count(self) -> int:
        u = ctypes.c_uint64()
        check(N.lib().mg_device_counters(self._h, ctypes.byref(u), None))
        return u.value

    def download_count(self) -> int:
        d = ctypes.c_uint64()
        check(N.lib().mg_device_counters(self._h, None, ctypes.byref(d)))
        return d.value

    def launch_count(self) -> int:
        return int(N.lib().mg_device_launch_count(self._h))

    # ---- buffers --------------------------------------------------------------------
    def _new(self, fn, dtype, shape) -> DeviceBuffer:
        out = ctypes.c_void_p()
        check(fn(self._h, _dtype_code(dtype), len(shape), N.shape_array(shape), ctypes.byref(out)))
        return DeviceBuffer(out.value, self)

    def empty(self, shape, dtype="f32") -> DeviceBuffer:
        return self._new(N.lib().mg_buffer_create, dtype, shape)

    def zeros(self, shape, dtype="f32") -> DeviceBuffer:
        """``CudaKernels::zeros``: set on the device, no upload."""
        return self._new(N.lib().mg_buffer_zeros, dtype, shape)

    def upload(self, array, dtype="f32") -> DeviceBuffer:
        """f32 host values to a new device buffer; f16/bf16 are encoded with the
        reference's RNE rules (``upload`` / ``upload_half``)."""
        a = np.ascontiguousarray(array, dtype=np.float32)
        buf = self.empty(a.shape, dtype)
        check(N.lib().mg_buffer_upload_f32(buf.handle, a.ctypes.data, a.size))
        return buf

    def upload_raw(self, array, dtype) -> DeviceBuffer:
        """Host bytes already in ``dtype`` (u16 bit patterns for f16/bf16)."""
        np_dtype = np.float32 if _dtype_code(dtype) == N.F32 else np.uint16
        a = np.ascontiguousarray(array, dtype=np_dtype)
        buf = self.empty(a.shape, dtype)
        check(N.lib().mg_buffer_upload(buf.handle, a.ctypes.data, a.nbytes))
        return buf

    def upload_q8_0(self, blocks, stored_rows: int, stored_cols: int, transposed: bool = True) -> DeviceBuffer:
        """``upload_packed_weight`` for ``Q8_0``: 34-byte blocks (f16 scale, 32 int8 quants) of a
        [stored_rows, stored_cols] matrix; the logical matrix is its transpose when ``transposed``."""
        raw = np.ascontiguousarray(np.frombuffer(bytes(blocks), np.uint8) if isinstance(blocks, (bytes, bytearray))
                                   else np.asarray(blocks, np.uint8).ravel())
        out = ctypes.c_void_p()
        check(N.lib().mg_buffer_upload_q8_0(self._h, raw.ctypes.data, raw.nbytes, stored_rows, stored_cols,
                                            1 if transposed else 0, ctypes.byref(out)))
        return DeviceBuffer(out.value, self)

    def dequantize_q8(self, packed, out=None):
        """``dequantize_q8``: a packed weight's logical matrix as f32."""
        return self._run(N.lib().mg_dequantize_q8, packed.handle, out=out)

    def download(self, buf: DeviceBuffer) -> np.ndarray:
        """Values as f32 (half buffers decoded exactly, packed weights dequantized)."""
        out = np.empty(buf.shape, dtype=np.float32)
        check(N.lib().mg_buffer_download_f32(buf.handle, out.ctypes.data, out.size))
        return out

    def download_raw(self, buf: DeviceBuffer) -> np.ndarray:
        np_dtype = np.float32 if buf.dtype == "f32" else np.uint16
        out = np.empty(buf.shape, dtype=np_dtype)
        check(N.lib().mg_buffer_download(buf.handle, out.ctypes.data, out.nbytes))
        return out

    def download_rows(self, buf: DeviceBuffer, first_row: int, rows: int) -> Optional[np.ndarray]:
        """Rows of a rank-2 f32 buffer; None when the range is outside it."""
        shape = buf.shape
        if len(shape) != 2 or first_row + rows > shape[0]:
            return None
        out = np.empty((rows, shape[1]), dtype=np.float32)
        check(N.lib().mg_buffer_download_rows(buf.handle, first_row, rows, out.ctypes.data, out.size))
        return out

    def wrap(self, ptr: int, shape, dtype="f32", owner=None) -> DeviceBuffer:
        """A non-owning view of existing device memory (e.g. a torch tensor)."""
        out = ctypes.c_void_p()
        check(N.lib().mg_buffer_wrap(self._h, _dtype_code(dtype), len(shape), N.shape_array(shape),
                                     ctypes.c_void_p(ptr), ctypes.byref(out)))
        return DeviceBuffer(out.value, self, owner)

    def wrap_tensor(self, t) -> DeviceBuffer:
        """A view of a contiguous CUDA torch tensor (f32, f16 or bf16) without a copy."""
        import torch
        if not t.is_cuda or not t.is_contiguous():
            raise CudaError(3, "only contiguous CUDA tensors can be wrapped")
        dt = {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}[t.dtype]
        return self.wrap(t.data_ptr(), tuple(t.shape), dt, owner=t)

    # ---- kernels ----------------------------------------------------------------------
    def _run(self, fn, *args, out: Optional[DeviceBuffer] = None) -> DeviceBuffer:
        o = ctypes.c_void_p(out.handle.value if out is not None else None)
        check(fn(self._h, *args, ctypes.byref(o)))
        if out is not None and o.value == out.handle.value:
            return out
        return DeviceBuffer(o.value, self)

    def add(self, a, b, out=None):
        return self._run(N.lib().mg_add, a.handle, b.handle, out=out)

    def mul(self, a, b, out=None):
        return self._run(N.lib().mg_mul, a.handle, b.handle, out=out)

    def residual_add(self, x, residual, out=None):
        return self._run(N.lib().mg_residual_add, x.handle, residual.handle, out=out)

    def scale(self, x, factor: float, out=None):
        return self._run(N.lib().mg_scale, x.handle, ctypes.c_float(factor), out=out)

    def silu(self, x, out=None):
        return self._run(N.lib().mg_silu, x.handle, out=out)

    def silu_mul(self, gate, up, out=None):
        return self._run(N.lib().mg_silu_mul, gate.handle, up.handle, out=out)

    def add_half(self, a, b, out=None):
        return self._run(N.lib().mg_add_half, a.handle, b.handle, out=out)

    def mul_half(self, a, b, out=None):
        return self._run(N.lib().mg_mul_half, a.handle, b.handle, out=out)

    def half_binary_f32(self, a, b, dtype: str, op: str, out=None):
        return self._run(N.lib().mg_half_binary_f32, a.handle, b.handle, _dtype_code(dtype),
                         0 if op == "add" else 1, out=out)

    def embedding_lookup(self, table, ids, scale: Optional[float] = None, out=None):
        return self._run(N.lib().mg_embedding, table.handle, ids.handle, 0 if scale is None else 1,
                         ctypes.c_float(scale or 0.0), out=out)

    def rmsnorm(self, x, weight=None, epsilon: float = 1e-6, heads=None, out=None):
        hc, hd = heads if heads else (0, 0)
        return self._run(N.lib().mg_rmsnorm, x.handle, weight.handle if weight is not None else None,
                         ctypes.c_float(epsilon), hc, hd, out=out)

    def rope(self, x, base=10000.0, scale=1.0, dimension=None, position_offset=0, head_count=1,
             pairing="interleaved", banded=None, yarn=None, rotated_pairs=None, out=None):
        """``rope_scaled``: ``banded`` = (factor, low, high, original_context_length);
        ``yarn`` = (factor, correction_low, correction_high, attention_factor)."""
        p = N.RopeParams()
        p.base, p.scale = base, scale
        cols = x.shape[-1]
        p.dimension = dimension if dimension is not None else cols // max(1, head_count)
        p.position_offset, p.head_count = position_offset, head_count
        p.pairing = {"interleaved": 0, "half_split": 1}[pairing]
        if banded:
            p.banded_factor, p.low_freq_factor, p.high_freq_factor, p.original_context_length = banded
        p.amplitude = 1.0
        if yarn:
            p.yarn_factor, p.yarn_low, p.yarn_high, p.amplitude = yarn
        p.rotated_pairs = (2 ** 64 - 1) if rotated_pairs is None else rotated_pairs
        return self._run(N.lib().mg_rope, x.handle, ctypes.byref(p), out=out)

    def softmax_rows(self, x, out=None):
        return self._run(N.lib().mg_softmax, x.handle, out=out)

    def greedy_select(self, logits, row: int, excluded=(), temperature: float = 0.0) -> Optional[int]:
        """``greedy_select``: the column of logits row ``row`` with the highest finite score /
        temperature outside the ``excluded`` ``(start, end)`` ranges, ties to the lowest column;
        None when no column is eligible."""
        found, column = ctypes.c_int(), ctypes.c_uint64()
        pairs, count = N.range_pairs(excluded)
        check(N.lib().mg_greedy_select(self.handle, logits.handle, row, pairs, count, ctypes.c_float(temperature),
                                       ctypes.byref(found), ctypes.byref(column)))
        return int(column.value) if found.value else None

    def gelu_tanh(self, x, out=None):
        """``gelu_tanh`` (the tanh approximation)."""
        return self._run(N.lib().mg_gelu_tanh, x.handle, out=out)

    def sigmoid(self, x, out=None):
        return self._run(N.lib().mg_sigmoid, x.handle, out=out)

    def softcap(self, x, cap, out=None):
        """``cap * tanh(x / cap)``."""
        return self._run(N.lib().mg_softcap, x.handle, float(cap), out=out)

    def row_scale(self, x, scale, out=None):
        """``out[t, :] = x[t, :] * scale[t]``."""
        return self._run(N.lib().mg_row_scale, x.handle, scale.handle, out=out)

    def concat(self, a, b, out=None):
        """Along the first dimension."""
        return self._run(N.lib().mg_concat, a.handle, b.handle, out=out)

    def concat_heads(self, a, b, head_count, second_head_count=None, out=None):
        shc = head_count if second_head_count is None else second_head_count
        return self._run(N.lib().mg_concat_heads, a.handle, b.handle, int(head_count), int(shc), out=out)

    def batched_matmul(self, a, b, groups, transpose_b=False, out=None):
        return self._run(N.lib().mg_batched_matmul, a.handle, b.handle, int(groups), int(bool(transpose_b)), out=out)

    def kv_write(self, store, rows, row_offset):
        """``kv_write``: ``rows`` over ``store``'s rows ``row_offset..`` in place."""
        check(N.lib().mg_kv_write(self._h, store.handle, rows.handle, int(row_offset)))
        return store

    def matmul(self, a, b, transpose_a=False, transpose_b=False, out=None):
        return self._run(N.lib().mg_matmul, a.handle, b.handle, int(transpose_a), int(transpose_b), out=out)

    def matmul_bias(self, a, b, bias, transpose_a=False, transpose_b=False, out=None):
        return self._run(N.lib().mg_matmul_bias, a.handle, b.handle, bias.handle, int(transpose_a),
                         int(transpose_b), out=out)

    def matmul_residual(self, a, b, residual, transpose_a=False, transpose_b=False, out=None):
        return self._run(N.lib().mg_matmul_residual, a.handle, b.handle, residual.handle,
                         int(transpose_a), int(transpose_b), out=out)

    def gated_matmul(self, a, gate, up, transpose_a=False, transpose_b=False, out=None):
        return self._run(N.lib().mg_gated_matmul, a.handle, gate.handle, up.handle, int(transpose_a),
                         int(transpose_b), out=out)

    def attention(self, q, k, v, head_count, head_dimension, kv_head_count=None, window_size=None,
                  causal=False, key_count=None, scale=None, value_dimension=None, out=None):
        """``attention_valued`` (``src/kernels.rs:6505``)."""
        p = N.AttentionParams()
        p.head_count, p.head_dimension = head_count, head_dimension
        p.kv_head_count = kv_head_count or 0
        p.value_dimension = value_dimension or 0
        p.window_size = -1 if window_size is None else int(window_size)
        p.causal = int(bool(causal))
        p.key_count = -1 if key_count is None else int(key_count)
        p.has_scale = 0 if scale is None else 1
        p.scale = 0.0 if scale is None else float(scale)
        return self._run(N.lib().mg_attention, q.handle, k.handle, v.handle, ctypes.byref(p), out=out)
