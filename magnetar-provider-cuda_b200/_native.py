"""ctypes binding of ``libmagnetar_cuda.so`` (declared in ``include/magnetar_cuda.h``).

This is the same binding a Rust ``extern "C"`` block would make: opaque handles, plain
pointers and sizes, an ``mg_status`` return code.  There is no CPU fallback: when the
library is missing every entry point raises instead of computing anything.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libmagnetar_cuda.so")
CSRC = os.path.join(_HERE, "csrc")

MG_MAX_RANK = 8
F32, F16, BF16, Q8_0 = 0, 1, 2, 3
PACKED_Q8_0 = 0
ATTR_INT, ATTR_FLOAT, ATTR_BOOL, ATTR_STRING = 0, 1, 2, 3

# mg_status -> the reference's CudaErrorCode / KernelError names (src/error.rs:14-42).
STATUS_NAMES = {
    0: "Ok", 1: "ShapeUnsupported", 2: "DTypeUnsupported", 3: "LayoutUnsupported",
    4: "ExecutionFailed", 5: "OutOfDeviceMemory", 6: "CompilationFailed", 7: "DriverFailed",
    8: "DeviceUnavailable", 9: "CaptureUnsupported", 10: "KernelNotFound",
    11: "KernelAttributeUnsupported", 12: "InvalidArgument", 13: "KernelTimeout",
}


class CudaError(RuntimeError):
    """A failed call: ``code`` is the status name, ``detail`` the redacted diagnostic."""

    def __init__(self, status: int, detail: str):
        self.status = status
        self.code = STATUS_NAMES.get(status, f"Status{status}")
        self.detail = detail
        super().__init__(f"{self.code}: {detail}")


class RopeParams(ctypes.Structure):
    _fields_ = [
        ("base", ctypes.c_float), ("scale", ctypes.c_float),
        ("dimension", ctypes.c_uint64), ("position_offset", ctypes.c_uint64),
        ("head_count", ctypes.c_uint64), ("pairing", ctypes.c_int),
        ("banded_factor", ctypes.c_float), ("low_freq_factor", ctypes.c_float),
        ("high_freq_factor", ctypes.c_float), ("original_context_length", ctypes.c_float),
        ("rotated_pairs", ctypes.c_uint64),
        ("yarn_factor", ctypes.c_float), ("yarn_low", ctypes.c_float),
        ("yarn_high", ctypes.c_float), ("amplitude", ctypes.c_float),
    ]


class AttentionParams(ctypes.Structure):
    _fields_ = [
        ("head_count", ctypes.c_uint64), ("head_dimension", ctypes.c_uint64),
        ("kv_head_count", ctypes.c_uint64), ("value_dimension", ctypes.c_uint64),
        ("window_size", ctypes.c_int64), ("causal", ctypes.c_int),
        ("key_count", ctypes.c_int64), ("has_scale", ctypes.c_int), ("scale", ctypes.c_float),
    ]


class DeviceInfo(ctypes.Structure):
    _fields_ = [
        ("ordinal", ctypes.c_int), ("name", ctypes.c_char * 96),
        ("sm_major", ctypes.c_int), ("sm_minor", ctypes.c_int), ("sm_count", ctypes.c_int),
        ("total_bytes", ctypes.c_uint64), ("free_bytes", ctypes.c_uint64),
    ]


class Attribute(ctypes.Structure):
    _fields_ = [
        ("name", ctypes.c_char_p), ("kind", ctypes.c_int), ("int_value", ctypes.c_int64),
        ("float_value", ctypes.c_double), ("string_value", ctypes.c_char_p),
    ]


class Invocation(ctypes.Structure):
    _fields_ = [
        ("kernel", ctypes.c_char_p), ("input_count", ctypes.c_int),
        ("inputs", ctypes.POINTER(ctypes.c_char_p)), ("input_dtypes", ctypes.POINTER(ctypes.c_int)),
        ("output", ctypes.c_char_p), ("attribute_count", ctypes.c_int),
        ("attributes", ctypes.POINTER(Attribute)), ("deadline_millis", ctypes.c_int64),
    ]


_P = ctypes.c_void_p
_PP = ctypes.POINTER(ctypes.c_void_p)
_U64 = ctypes.c_uint64
_U64P = ctypes.POINTER(ctypes.c_uint64)
_I = ctypes.c_int
_IP = ctypes.POINTER(ctypes.c_int)
_F = ctypes.c_float
_S = ctypes.c_char_p

# name -> argtypes (every function returns mg_status unless listed in _RESTYPES)
SIGNATURES = {
    "mg_abi_version": [],
    "mg_last_error": [],
    "mg_status_name": [_I],
    "mg_device_count": [_IP],
    "mg_device_open": [_I, _PP],
    "mg_device_close": [_P],
    "mg_device_get_info": [_P, ctypes.POINTER(DeviceInfo)],
    "mg_device_synchronize": [_P],
    "mg_device_stream": [_P],
    "mg_device_set_stream": [_P, _P],
    "mg_device_counters": [_P, _U64P, _U64P],
    "mg_device_launch_count": [_P],
    "mg_buffer_create": [_P, _I, _I, _U64P, _PP],
    "mg_buffer_zeros": [_P, _I, _I, _U64P, _PP],
    "mg_buffer_wrap": [_P, _I, _I, _U64P, _P, _PP],
    "mg_buffer_release": [_P],
    "mg_buffer_upload": [_P, _P, _U64],
    "mg_buffer_download": [_P, _P, _U64],
    "mg_buffer_upload_f32": [_P, _P, _U64],
    "mg_buffer_download_f32": [_P, _P, _U64],
    "mg_buffer_download_rows": [_P, _U64, _U64, _P, _U64],
    "mg_buffer_shape": [_P, _IP, _U64P],
    "mg_buffer_dtype": [_P, _IP],
    "mg_buffer_reshape": [_P, _I, _U64P],
    "mg_buffer_device_ptr": [_P],
    "mg_buffer_set_weight": [_P, _I],
    "mg_buffer_is_compact": [_P],
    "mg_buffer_upload_q8_0": [_P, _P, _U64, _U64, _U64, _I, _PP],
    "mg_buffer_is_q8": [_P],
    "mg_dequantize_q8": [_P, _P, _PP],
    "mg_add": [_P, _P, _P, _PP],
    "mg_mul": [_P, _P, _P, _PP],
    "mg_residual_add": [_P, _P, _P, _PP],
    "mg_scale": [_P, _P, _F, _PP],
    "mg_silu": [_P, _P, _PP],
    "mg_silu_mul": [_P, _P, _P, _PP],
    "mg_add_half": [_P, _P, _P, _PP],
    "mg_mul_half": [_P, _P, _P, _PP],
    "mg_half_binary_f32": [_P, _P, _P, _I, _I, _PP],
    "mg_embedding": [_P, _P, _P, _I, _F, _PP],
    "mg_rmsnorm": [_P, _P, _P, _F, _U64, _U64, _PP],
    "mg_rope": [_P, _P, ctypes.POINTER(RopeParams), _PP],
    "mg_softmax": [_P, _P, _PP],
    "mg_greedy_select": [_P, _P, _U64, _U64P, ctypes.c_uint32, _F, _IP, _U64P],
    "mg_kv_write": [_P, _P, _P, _U64],
    "mg_gelu_tanh": [_P, _P, _PP],
    "mg_sigmoid": [_P, _P, _PP],
    "mg_softcap": [_P, _P, _F, _PP],
    "mg_row_scale": [_P, _P, _P, _PP],
    "mg_concat": [_P, _P, _P, _PP],
    "mg_concat_heads": [_P, _P, _P, _U64, _U64, _PP],
    "mg_batched_matmul": [_P, _P, _P, _U64, _I, _PP],
    "mg_matmul": [_P, _P, _P, _I, _I, _PP],
    "mg_matmul_bias": [_P, _P, _P, _P, _I, _I, _PP],
    "mg_matmul_residual": [_P, _P, _P, _P, _I, _I, _PP],
    "mg_gated_matmul": [_P, _P, _P, _P, _I, _I, _PP],
    "mg_matmul_gemv_fixed": [_I, _P, _P, _P, _P, _U64, _U64, _U64],
    "mg_attention": [_P, _P, _P, _P, ctypes.POINTER(AttentionParams), _PP],
    "mg_executor_create": [_P, _PP],
    "mg_executor_destroy": [_P],
    "mg_executor_write_tensor": [_P, _S, _I, _U64P, _P],
    "mg_executor_write_weight_tensor": [_P, _S, _I, _U64P, _P],
    "mg_executor_write_zeroed_tensor": [_P, _S, _I, _U64P],
    "mg_executor_adopt_buffer": [_P, _S, _P],
    "mg_executor_buffer": [_P, _S, _PP],
    "mg_executor_read_tensor": [_P, _S, _P, _U64, _IP, _U64P],
    "mg_executor_read_tensor_rows": [_P, _S, _U64, _U64, _P, _U64],
    "mg_executor_write_packed_weight_tensor": [_P, _S, _I, _P, _U64, _U64, _U64, _I],
    "mg_executor_select_greedy_column": [_P, _S, _U64, _U64P, ctypes.c_uint32, _F, _IP, _U64P],
    "mg_executor_release_tensor": [_P, _S, _IP],
    "mg_executor_resident_shape": [_P, _S, _IP, _IP, _U64P],
    "mg_executor_copy_tensor": [_P, _S, _S],
    "mg_executor_submit_kernel": [_P, ctypes.POINTER(Invocation)],
    "mg_executor_synchronize": [_P],
    "mg_executor_begin_step_capture": [_P],
    "mg_executor_begin_step_capture_advancing": [_P, ctypes.POINTER(ctypes.c_char_p), _I],
    "mg_executor_replay_step_at": [_P, _U64],
    "mg_executor_replay_step_io": [_P, _U64, _P, _I],
    "mg_executor_step_max_offset": [_P, _U64P],
    "mg_executor_end_step_capture": [_P],
    "mg_executor_abort_step_capture": [_P],
    "mg_executor_replay_step": [_P],
    "mg_executor_replay_steps": [_P, _I],
    "mg_executor_launch_step": [_P],
    "mg_executor_check_steps": [_P],
    "mg_executor_observations": [_P, _U64P, _U64P, _U64P],
    "mg_executor_observation_log": [_P, _P, ctypes.c_uint32, ctypes.POINTER(ctypes.c_uint32)],
    "mg_executor_end_step_capture_id": [_P, _U64P],
    "mg_executor_replay_capture": [_P, _U64, _U64, _P, _I],
    "mg_executor_release_step_capture": [_P, _U64],
    "mg_executor_step_capture_count": [_P, _IP],
    "mg_comm_unique_id": [ctypes.c_char_p],
    "mg_comm_init": [_P, _I, _I, ctypes.c_char_p, _PP],
    "mg_comm_destroy": [_P],
    "mg_comm_all_reduce": [_P, _P],
    "mg_comm_set_timeout": [_P, ctypes.c_int64],
    "mg_comm_check": [_P],
    "mg_comm_wait": [_P, ctypes.c_int64],
    "mg_comm_abort": [_P],
    "mg_comm_is_aborted": [_P],
    "mg_comm_set_mlp_timing": [_P, ctypes.c_int],
    "mg_comm_mlp_timing": [_P, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_float)],
    "mg_comm_settle_selftest": [_IP, _I, ctypes.c_int64, _IP, _IP],
    "mg_tp_share": [_U64, _I, _I, _U64P, _U64P],
    "mg_tp_mlp": [_P, _P, _P, _P, _P, _I, _PP],
    "mg_executor_attach_comm": [_P, _P],
    "mg_executor_apply_tensor_parallel": [_P, _I, ctypes.POINTER(ctypes.c_char_p), _IP],
}

_RESTYPES = {
    "mg_abi_version": ctypes.c_int,
    "mg_last_error": ctypes.c_char_p,
    "mg_status_name": ctypes.c_char_p,
    "mg_device_stream": ctypes.c_void_p,
    "mg_device_launch_count": ctypes.c_uint64,
    "mg_buffer_device_ptr": ctypes.c_void_p,
    "mg_comm_is_aborted": ctypes.c_int,
}

_lib = None


def build(force: bool = False) -> str:
    """Compiles the native library for sm_100a with the committed Makefile (nvcc)."""
    jobs = str(max(1, min(16, os.cpu_count() or 1)))
    if force:
        subprocess.run(["make", "-C", CSRC, "clean"], check=True, stdout=subprocess.DEVNULL)
    subprocess.run(["make", "-C", CSRC, "-j", jobs], check=True, stdout=subprocess.DEVNULL)
    return LIB_PATH


OBSERVATION_KINDS = {0: "KernelDispatchStarted", 1: "KernelDispatchCompleted", 2: "KernelDispatchFailed",
                     3: "KernelTimeout", 4: "KernelMemoryFeasibilityFailed"}
OBSERVATION_LOG_CAPACITY = 4096


class Observation(ctypes.Structure):
    """mg_observation: one KernelObservation of the executor's log."""
    _fields_ = [("kind", ctypes.c_int), ("kernel", ctypes.c_char * 48), ("invocation", ctypes.c_uint64),
                ("status", ctypes.c_int)]


class StepIO(ctypes.Structure):
    """mg_step_io: one host input (to_device 1) or output (0) of a replay."""
    _fields_ = [("id", ctypes.c_char_p), ("host", ctypes.c_void_p), ("bytes", ctypes.c_uint64),
                ("to_device", ctypes.c_int)]


def range_pairs(ranges):
    """(start, end) ranges as a [2 * count] uint64 array for the C ABI, and the count."""
    flat = [int(v) for r in ranges for v in (r[0], r[1])]
    arr = (ctypes.c_uint64 * max(1, len(flat)))(*flat)
    return arr, len(flat) // 2


def _preload_nccl() -> None:
    """Loads the NCCL that ships with the framework's wheels (nvidia-nccl), when present, before
    this library: the library links libnccl.so.2 by its soname, and a process that later imports
    torch must find the NCCL torch was built against already loaded, not an older system copy
    this library happened to pull in first."""
    try:
        import importlib.util
        spec = importlib.util.find_spec("nvidia.nccl")
    except (ImportError, ValueError):
        return
    for root in (spec.submodule_search_locations or []) if spec else []:
        path = os.path.join(root, "lib", "libnccl.so.2")
        if os.path.exists(path):
            ctypes.CDLL(path, mode=ctypes.RTLD_GLOBAL)
            return


def lib():
    """The loaded library; raises (never falls back) when it is not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise CudaError(6, f"native library missing at {LIB_PATH}: run __graft_entry__.build()")
        _preload_nccl()
        L = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = _RESTYPES.get(name, ctypes.c_int)
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != 0:
        detail = lib().mg_last_error()
        raise CudaError(status, detail.decode() if detail else "")


def shape_array(shape):
    arr = (ctypes.c_uint64 * max(1, len(shape)))(*[int(s) for s in shape])
    return arr
