"""TEST INFRASTRUCTURE ONLY: numpy/ctypes front end of the C oracle (``liboracle.so``).

The oracle is the CPU restatement of the reference provider's hot-path kernels
(``src/kernels.cu`` of astorise/Magnetar-provider-CUDA); each wrapper names the reference
lines it follows.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
legs may import this module -- it checks and times, it is never the product path.
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_u64 = ctypes.c_uint64


class RopeParams(ctypes.Structure):
    _fields_ = [
        ("base", ctypes.c_float), ("scale", ctypes.c_float),
        ("dimension", _u64), ("position_offset", _u64), ("head_count", _u64),
        ("half_split", ctypes.c_uint32),
        ("banded_factor", ctypes.c_float), ("low_freq_factor", ctypes.c_float),
        ("high_freq_factor", ctypes.c_float), ("original_context_length", ctypes.c_float),
        ("rotated_pairs", _u64),
        ("yarn_factor", ctypes.c_float), ("yarn_low", ctypes.c_float),
        ("yarn_high", ctypes.c_float), ("amplitude", ctypes.c_float),
    ]


class AttentionParams(ctypes.Structure):
    _fields_ = [
        ("seq_len", _u64), ("kv_seq_len", _u64), ("head_count", _u64),
        ("kv_head_count", _u64), ("head_dimension", _u64),
        ("q_model_dim", _u64), ("kv_model_dim", _u64),
        ("causal", ctypes.c_int), ("window_size", ctypes.c_int64),
        ("query_position_offset", _u64), ("score_scale", ctypes.c_float),
        ("value_dimension", _u64), ("v_model_dim", _u64),
    ]


def build() -> str:
    """Compiles ``liboracle.so`` with the committed Makefile when it is missing or stale."""
    src = os.path.join(_HERE, "oracle.c")
    if (not os.path.exists(_LIB_PATH)
            or os.path.getmtime(_LIB_PATH) < max(os.path.getmtime(src),
                                                 os.path.getmtime(os.path.join(_HERE, "oracle.h")))):
        subprocess.run(["make", "-C", _HERE, "liboracle.so"], check=True,
                       stdout=subprocess.DEVNULL)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        L.orc_f16_to_f32.restype = ctypes.c_float
        L.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.orc_bf16_to_f32.restype = ctypes.c_float
        L.orc_bf16_to_f32.argtypes = [ctypes.c_uint16]
        L.orc_f32_to_f16.restype = ctypes.c_uint16
        L.orc_f32_to_f16.argtypes = [ctypes.c_float]
        L.orc_f32_to_bf16.restype = ctypes.c_uint16
        L.orc_f32_to_bf16.argtypes = [ctypes.c_float]
        L.orc_get_threads.restype = ctypes.c_int
        L.orc_greedy_select.restype = ctypes.c_int64
        L.orc_greedy_select.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_float]
        L.orc_embedding.restype = ctypes.c_int
        L.orc_softmax_rows.restype = ctypes.c_int
        _lib = L
    return _lib


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def threads() -> int:
    return int(lib().orc_get_threads())


def _f(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a, a.ctypes.data_as(_f32p)


def _u(a):
    a = np.ascontiguousarray(a, dtype=np.uint16)
    return a, a.ctypes.data_as(_u16p)


def _out(shape, dtype=np.float32):
    o = np.empty(shape, dtype=dtype)
    return o, o.ctypes.data_as(_u16p if dtype == np.uint16 else _f32p)


# ---- half precision: src/half_precision.rs:14-125 ------------------------------------

def f16_to_f32(bits: int) -> float:
    return lib().orc_f16_to_f32(bits)


def f32_to_f16(v: float) -> int:
    return lib().orc_f32_to_f16(v)


def bf16_to_f32(bits: int) -> float:
    return lib().orc_bf16_to_f32(bits)


def f32_to_bf16(v: float) -> int:
    return lib().orc_f32_to_bf16(v)


_DTYPE = {"f16": 1, "bf16": 2}
_OP = {"add": 0, "mul": 1}


def half_binary(a16, b16, dtype: str, op: str):
    """src/kernels.cu:2913-2939 on u16 bit patterns."""
    a, ap = _u(a16)
    b, bp = _u(b16)
    o, op_ = _out(a.shape, np.uint16)
    lib().orc_half_binary(ap, bp, op_, _u64(a.size), _DTYPE[dtype], _OP[op])
    return o


def half_binary_f32(a, b, dtype: str, op: str):
    """src/executor.rs:1970-2013: f32 values in, encoded, half op, decoded back to f32."""
    a, ap = _f(a)
    b, bp = _f(b)
    o, op_ = _out(a.shape)
    lib().orc_half_binary_f32(ap, bp, op_, _u64(a.size), _DTYPE[dtype], _OP[op])
    return o


def encode_half(x, dtype: str):
    """f32 -> half bits with the reference's RNE and NaN rules (src/half_precision.rs:48-117);
    bit patterns (NaN payloads included) pass through C unchanged."""
    x, xp = _f(x)
    o, op = _out(x.shape, np.uint16)
    lib().orc_encode_half(xp, op, _u64(x.size), _DTYPE[dtype])
    return o


def decode_half(bits, dtype: str):
    """half bits -> f32, exactly (src/half_precision.rs:15-44)."""
    b, bp = _u(bits)
    o, op = _out(b.shape)
    lib().orc_decode_half(bp, op, _u64(b.size), _DTYPE[dtype])
    return o


# ---- elementwise: src/kernels.cu:30-117, 1091-1096 -----------------------------------

def add(a, b):
    a, ap = _f(a)
    b, bp = _f(b)
    if a.shape == b.shape:
        o, op = _out(a.shape)
        lib().orc_add(ap, bp, op, _u64(a.size))
        return o
    cols = a.shape[-1]
    o, op = _out(a.shape)
    lib().orc_bias_add(ap, bp, op, _u64(cols), _u64(a.size))
    return o


def mul(a, b):
    a, ap = _f(a)
    b, bp = _f(b)
    o, op = _out(a.shape)
    if b.size == 1 and a.shape != b.shape:
        lib().orc_mul_scalar(ap, bp, op, _u64(a.size))
    else:
        lib().orc_mul(ap, bp, op, _u64(a.size))
    return o


def scale(x, factor):
    x, xp = _f(x)
    o, op = _out(x.shape)
    lib().orc_scale(xp, op, ctypes.c_float(factor), _u64(x.size))
    return o


def silu(x):
    x, xp = _f(x)
    o, op = _out(x.shape)
    lib().orc_silu(xp, op, _u64(x.size))
    return o


def gelu_tanh(x):
    """src/kernels.cu:80-92"""
    x, xp = _f(x)
    o, op = _out(x.shape)
    lib().orc_gelu_tanh(xp, op, _u64(x.size))
    return o


def sigmoid(x):
    """src/kernels.cu:1079-1084"""
    x, xp = _f(x)
    o, op = _out(x.shape)
    lib().orc_sigmoid(xp, op, _u64(x.size))
    return o


def softcap(x, cap):
    """src/kernels.cu:103-109"""
    x, xp = _f(x)
    o, op = _out(x.shape)
    lib().orc_softcap(xp, op, ctypes.c_float(cap), _u64(x.size))
    return o


def row_scale(x, scale):
    """src/kernels.cu:1066-1077"""
    x, xp = _f(x)
    s, sp = _f(scale)
    o, op = _out(x.shape)
    lib().orc_row_scale(xp, sp, op, _u64(x.shape[0]), _u64(x.shape[1]))
    return o


def q8_0_dequantize(blocks, stored_rows, stored_cols, transposed=True):
    """src/kernels.rs:1800-1838 + src/kernels.cu:230-246: the logical f32 matrix of Q8_0 blocks"""
    raw = np.ascontiguousarray(np.asarray(blocks, np.uint8).ravel())
    assert raw.size == stored_rows * stored_cols // 32 * 34
    shape = (stored_cols, stored_rows) if transposed else (stored_rows, stored_cols)
    o, op = _out(shape)
    lib().orc_q8_0_dequantize(raw.ctypes.data_as(ctypes.c_void_p), _u64(stored_rows), _u64(stored_cols),
                              int(bool(transposed)), op)
    return o


def greedy_select(logits, row, excluded=(), temperature=0.0):
    """src/tests_conformance.rs:571-587 (host greedy selection); None when nothing is eligible"""
    x = np.ascontiguousarray(logits, np.float32)
    cols = x.shape[-1]
    r = np.ascontiguousarray(x.reshape(-1, cols)[row])
    pairs = np.ascontiguousarray(np.array([v for p in excluded for v in p] or [0, 0], np.uint64))
    c = lib().orc_greedy_select(r.ctypes.data, cols, pairs.ctypes.data, len(excluded), float(temperature))
    return None if c < 0 else int(c)


def concat(a, b):
    """src/kernels.rs:3058-3100: along the first dimension"""
    return np.concatenate([np.asarray(a, np.float32), np.asarray(b, np.float32)], axis=0)


def concat_heads(a, b, head_count, second_head_count=None):
    """src/kernels.cu:5786-5812"""
    a, ap = _f(a)
    b, bp = _f(b)
    second = head_count if second_head_count is None else second_head_count
    rows = a.shape[0]
    aw, bw = a.shape[1] // head_count, b.shape[1] // second
    o, op = _out((rows, head_count * (aw + bw)))
    lib().orc_concat_heads(ap, bp, op, _u64(rows), _u64(head_count), _u64(aw), _u64(bw), _u64(second))
    return o


def batched_matmul(a, b, groups, transpose_b=False):
    """src/kernels.cu:6296-6336"""
    a, ap = _f(a)
    b, bp = _f(b)
    rows, acols = a.shape
    k = acols // groups
    n = b.shape[0] // groups if transpose_b else b.shape[1]
    o, op = _out((rows, groups * n))
    lib().orc_batched_matmul(ap, bp, op, _u64(rows), _u64(groups), _u64(k), _u64(n), ctypes.c_int(int(transpose_b)))
    return o


def silu_mul(g, u):
    g, gp = _f(g)
    u, up = _f(u)
    o, op = _out(g.shape)
    lib().orc_silu_mul(gp, up, op, _u64(g.size))
    return o


# ---- embedding: src/kernels.cu:127-176 ------------------------------------------------

def embedding(table, ids, fill=np.nan):
    """Returns (rows, invalid_flag); rows of invalid ids keep ``fill``."""
    t, tp = _f(table)
    i, ip = _f(ids)
    vocab, dim = t.shape
    o = np.full((i.size, dim), fill, dtype=np.float32)
    flag = lib().orc_embedding(tp, ip, o.ctypes.data_as(_f32p), _u64(dim), _u64(i.size), _u64(vocab))
    return o, bool(flag)


# ---- rmsnorm: src/kernels.cu:1103-1138 ------------------------------------------------

def rmsnorm(x, weight=None, epsilon=1e-6, heads=None):
    x, xp = _f(x)
    cols = x.shape[-1] if heads is None else heads[1]
    rows = x.size // cols
    if weight is None:
        wp, stride = None, 0
    else:
        w, wp = _f(weight)
        stride = 0 if w.size == cols else cols
    o, op = _out(x.shape)
    lib().orc_rmsnorm(xp, wp, op, _u64(rows), _u64(cols), _u64(stride), ctypes.c_float(epsilon))
    return o


# ---- rope: src/kernels.cu:1147-1229 ---------------------------------------------------

def rope(x, base=10000.0, scale=1.0, dimension=None, position_offset=0, head_count=1,
         half_split=False, banded=None, yarn=None, rotated_pairs=None):
    """``banded`` = (factor, low_freq_factor, high_freq_factor, original_context_length);
    ``yarn`` = (factor, low, high, attention_factor), the correction range already computed."""
    x, xp = _f(x)
    rows, cols = x.shape
    p = RopeParams()
    p.base, p.scale = base, scale
    p.dimension = dimension if dimension is not None else cols // head_count
    p.position_offset, p.head_count, p.half_split = position_offset, head_count, int(half_split)
    half = p.dimension // 2
    if banded:
        p.banded_factor, p.low_freq_factor, p.high_freq_factor, p.original_context_length = banded
    p.rotated_pairs = half if rotated_pairs is None else min(rotated_pairs, half)
    p.amplitude = 1.0
    if yarn:
        p.yarn_factor, p.yarn_low, p.yarn_high, p.amplitude = yarn
    o, op = _out(x.shape)
    lib().orc_rope(xp, op, _u64(rows), _u64(cols), ctypes.byref(p))
    return o


# ---- softmax: src/kernels.cu:1232-1260 ------------------------------------------------

def softmax(x):
    x, xp = _f(x)
    rows, cols = x.shape
    o, op = _out(x.shape)
    flag = lib().orc_softmax_rows(xp, op, _u64(rows), _u64(cols))
    return o, bool(flag)


# ---- matmul: src/kernels.cu:1265-1294 -------------------------------------------------

def matmul(a, b, transpose_a=False, transpose_b=False, addend=None, addend_mode=0):
    a, ap = _f(a)
    b, bp = _f(b)
    m, k = (a.shape[1], a.shape[0]) if transpose_a else a.shape
    n = b.shape[0] if transpose_b else b.shape[1]
    o, op = _out((m, n))
    adp = None
    if addend is not None:
        ad, adp = _f(addend)
    lib().orc_matmul(ap, bp, op, _u64(m), _u64(k), _u64(n), int(transpose_a), int(transpose_b),
                     adp, int(addend_mode))
    return o


def gated_matmul(a, gate, up, transpose_a=False, transpose_b=False):
    a, ap = _f(a)
    g, gp = _f(gate)
    u, up_ = _f(up)
    m, k = (a.shape[1], a.shape[0]) if transpose_a else a.shape
    n = g.shape[0] if transpose_b else g.shape[1]
    o, op = _out((m, n))
    lib().orc_gated_matmul(ap, gp, up_, op, _u64(m), _u64(k), _u64(n), int(transpose_a),
                           int(transpose_b))
    return o


# ---- attention: src/kernels.cu:1873-1959, wrapper rules src/kernels.rs:6505-6629 -------

def attention(q, k, v, head_count, head_dimension, kv_head_count=None, window_size=None,
              causal=False, key_count=None, scale=None, value_dimension=None):
    q, qp = _f(q)
    k, kp = _f(k)
    v, vp = _f(v)
    kvh = kv_head_count or head_count
    vd = value_dimension or head_dimension
    seq = q.shape[0]
    kv_seq = key_count if key_count is not None else k.shape[0]
    p = AttentionParams()
    p.seq_len, p.kv_seq_len, p.head_count, p.kv_head_count = seq, kv_seq, head_count, kvh
    p.head_dimension, p.q_model_dim, p.kv_model_dim = head_dimension, q.shape[1], k.shape[1]
    p.causal = int(causal)
    p.window_size = -1 if window_size is None else int(window_size)
    p.query_position_offset = kv_seq - seq
    p.score_scale = 0.0 if scale is None else float(scale)
    p.value_dimension, p.v_model_dim = vd, v.shape[1]
    o, op = _out((seq, head_count * vd))
    lib().orc_attention(qp, kp, vp, op, ctypes.byref(p))
    return o


def rel_l2(actual, expected) -> float:
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    den = math.sqrt(float(np.sum(e * e)))
    num = math.sqrt(float(np.sum((a - e) ** 2)))
    return num / den if den > 0 else num
