"""TEST INFRASTRUCTURE ONLY: the reference's own per-op CUDA kernels, run on the GPU.

``oracle/_ref/kernels.ptx`` is compiled by ``oracle/Makefile`` (target ``ref``) from the
reference's ``src/kernels.cu`` where it lies, with the options the reference's NVRTC call uses
(no options: default architecture, FMA contraction on, no fast math; ``src/kernels.rs:807``).
This module loads that PTX through the CUDA driver API, exactly as the reference loads its
NVRTC output by kernel name (``src/kernels.rs:807-823``), and launches each kernel with the
launch shape and argument list of the reference's wrapper (cited per function).  It is used to
pin the CPU oracle (fixtures made by ``tests/golden/make_ref_golden.py``) and, in ``-m gpu``
tests, as a second checker of the provider's kernels.  Nothing in the package imports it.

Device memory comes from torch; every function takes and returns torch tensors on the current
device and synchronises before it returns.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
PTX_PATH = os.path.join(_HERE, "_ref", "kernels.ptx")

_cuda = None
_module = None
_functions = {}

# cudarc's LaunchConfig::for_num_elems: 1024 threads per block.
_THREADS = 1024
# src/kernels.rs:136-138
RMSNORM_THREADS = 256


def available() -> bool:
    return os.path.exists(PTX_PATH)


def _check(r, what):
    if r != 0:
        msg = ctypes.c_char_p()
        _cuda.cuGetErrorString(r, ctypes.byref(msg))
        raise RuntimeError(f"{what}: CUDA driver error {r} ({msg.value.decode() if msg.value else '?'})")


def _load():
    global _cuda, _module
    if _module is not None:
        return
    import torch
    if not available():
        raise FileNotFoundError(f"{PTX_PATH} is missing: run `make -C oracle ref` where the reference source is")
    torch.cuda.init()
    torch.empty(1, device="cuda")  # the primary context is current on this thread
    _cuda = ctypes.CDLL("libcuda.so.1")
    _check(_cuda.cuInit(0), "cuInit")
    with open(PTX_PATH, "rb") as f:
        image = f.read() + b"\0"
    mod = ctypes.c_void_p()
    _check(_cuda.cuModuleLoadData(ctypes.byref(mod), ctypes.c_char_p(image)), "loading the reference kernels")
    _module = mod


def _function(name):
    _load()
    f = _functions.get(name)
    if f is None:
        f = ctypes.c_void_p()
        _check(_cuda.cuModuleGetFunction(ctypes.byref(f), _module, name.encode()), f"function {name}")
        _functions[name] = f
    return f


def _u64(v):
    return ctypes.c_uint64(int(v))


def _ptr(t):
    return ctypes.c_uint64(0 if t is None else int(t.data_ptr()))


def _launch(name, grid, block, args, smem=0):
    import torch
    f = _function(name)
    params = (ctypes.c_void_p * len(args))(*[ctypes.cast(ctypes.byref(a), ctypes.c_void_p) for a in args])
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _check(_cuda.cuLaunchKernel(f, int(grid), 1, 1, int(block), 1, 1, int(smem), stream, params, None), f"launching {name}")
    torch.cuda.synchronize()


def _elems(n):
    return max(1, (int(n) + _THREADS - 1) // _THREADS)


def _f32(x):
    import torch
    return torch.as_tensor(x, dtype=torch.float32, device="cuda").contiguous()


# ---- elementwise: src/kernels.rs:2956-3118 (for_num_elems(n)) ----------------------------

def _binary(name, a, b):
    import torch
    a, b = _f32(a), _f32(b)
    out = torch.empty_like(a)
    _launch(name, _elems(a.numel()), _THREADS, [_ptr(a), _ptr(b), _ptr(out), _u64(a.numel())])
    return out


def add(a, b):
    """add_kernel, src/kernels.cu:30-36"""
    return _binary("add_kernel", a, b)


def mul(a, b):
    """mul_kernel, src/kernels.cu:55-61"""
    return _binary("mul_kernel", a, b)


def silu_mul(g, u):
    """silu_mul_kernel, src/kernels.cu:64-71"""
    return _binary("silu_mul_kernel", g, u)


def _unary(name, x):
    import torch
    x = _f32(x)
    out = torch.empty_like(x)
    _launch(name, _elems(x.numel()), _THREADS, [_ptr(x), _ptr(out), _u64(x.numel())])
    return out


def silu(x):
    """silu_kernel, src/kernels.cu:73-79"""
    return _unary("silu_kernel", x)


def gelu_tanh(x):
    """gelu_tanh_kernel, src/kernels.cu:88-94"""
    return _unary("gelu_tanh_kernel", x)


def sigmoid(x):
    """sigmoid_kernel, src/kernels.cu:1079-1084"""
    return _unary("sigmoid_kernel", x)


def half_binary(a16, b16, dtype, op):
    """add/mul_{f16,bf16}_kernel, src/kernels.cu:2913-2939 (16-bit patterns in int16 tensors)"""
    import torch
    a = torch.as_tensor(a16, device="cuda").view(torch.int16).contiguous()
    b = torch.as_tensor(b16, device="cuda").view(torch.int16).contiguous()
    out = torch.empty_like(a)
    _launch(f"{op}_{dtype}_kernel", _elems(a.numel()), _THREADS, [_ptr(a), _ptr(b), _ptr(out), _u64(a.numel())])
    return out


# ---- embedding: src/kernels.rs:3914-3928 -------------------------------------------------

def embedding(table, ids, fill=float("nan")):
    """embedding_lookup_kernel, src/kernels.cu:127-176: (rows, invalid flag); rows of invalid
    ids keep ``fill``"""
    import torch
    t, i = _f32(table), _f32(ids).reshape(-1)
    vocab, dim = t.shape
    out = torch.full((i.numel(), dim), fill, dtype=torch.float32, device="cuda")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    _launch("embedding_lookup_kernel", _elems(i.numel()), _THREADS,
            [_ptr(t), _ptr(i), _ptr(out), _u64(dim), _u64(i.numel()), _u64(vocab), _ptr(flag), _u64(0), _u64(0),
             _u64(0)])
    return out, bool(flag.item())


# ---- rmsnorm: src/kernels.rs:4082-4096 (grid rows, RMSNORM_THREADS) -----------------------

def rmsnorm(x, weight=None, epsilon=1e-6, heads=None):
    """rmsnorm_kernel, src/kernels.cu:1104-1138; ``heads`` = (head_count, head_dimension)
    normalises each head's slice with the gain repeated (stride 0) or per head"""
    import torch
    x = _f32(x)
    cols = x.shape[-1] if heads is None else heads[1]
    rows = x.numel() // cols
    if weight is None:
        w, stride = None, 0
    else:
        w = _f32(weight)
        stride = 0 if w.numel() == cols else cols
    out = torch.empty_like(x)
    _launch("rmsnorm_kernel", rows, RMSNORM_THREADS,
            [_ptr(x), _ptr(w), _ptr(out), _u64(rows), _u64(cols), _u64(stride), ctypes.c_float(epsilon)])
    return out


# ---- rope: src/kernels.rs:4290-4347 (for_num_elems(rows * heads * half)) ------------------

def rope(x, base=10000.0, scale=1.0, dimension=None, position_offset=0, head_count=1, half_split=False,
         banded=None, yarn=None, rotated_pairs=None):
    """rope_kernel, src/kernels.cu:1147-1229, with the oracle's argument conventions"""
    x = _f32(x)
    rows, cols = x.shape
    dim = dimension if dimension is not None else cols // head_count
    half = dim // 2
    out = x.clone()  # columns past `dimension` pass through (src/kernels.rs:4317-4323)
    bf, lo, hi, ocl = banded if banded else (0.0, 0.0, 0.0, 0.0)
    yf, yl, yh, amp = yarn if yarn else (0.0, 0.0, 0.0, 1.0)
    rp = half if rotated_pairs is None else min(rotated_pairs, half)
    F = ctypes.c_float
    _launch("rope_kernel", _elems(rows * head_count * half), _THREADS,
            [_ptr(x), _ptr(out), _u64(rows), _u64(cols), _u64(half), F(base), F(scale), _u64(dim),
             _u64(position_offset), _u64(head_count), ctypes.c_uint32(int(half_split)), _u64(0), F(bf), F(lo), F(hi),
             F(ocl), _u64(rp), F(yf), F(yl), F(yh), F(amp)])
    return out


# ---- softmax: src/kernels.rs:4357-4386 (for_num_elems(rows)) ------------------------------

def softmax(x):
    """softmax_rows_kernel, src/kernels.cu:1232-1260: (probabilities, non-finite-row flag)"""
    import torch
    x = _f32(x)
    rows, cols = x.shape
    out = torch.zeros_like(x)
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    _launch("softmax_rows_kernel", _elems(rows), _THREADS, [_ptr(x), _ptr(out), _u64(rows), _u64(cols), _ptr(flag)])
    return out, bool(flag.item())


# ---- matmul: src/kernels.rs:5544-5553, 5761-5775 (for_num_elems(m * n)) --------------------

def matmul(a, b, transpose_a=False, transpose_b=False):
    """matmul_kernel, src/kernels.cu:1265-1294: one thread per output, k ascending"""
    import torch
    a, b = _f32(a), _f32(b)
    a_rows, a_cols = a.shape
    b_rows, b_cols = b.shape
    m, k = (a_cols, a_rows) if transpose_a else (a_rows, a_cols)
    n = b_rows if transpose_b else b_cols
    a_row, a_inner = (1, a_cols) if transpose_a else (a_cols, 1)
    b_inner, b_col = (1, b_cols) if transpose_b else (b_cols, 1)
    out = torch.empty(m, n, dtype=torch.float32, device="cuda")
    _launch("matmul_kernel", _elems(m * n), _THREADS,
            [_ptr(a), _ptr(b), _ptr(out), _u64(m), _u64(k), _u64(n), _u64(a_row), _u64(a_inner), _u64(b_inner),
             _u64(b_col), _u64(0)])
    return out


# ---- attention: src/kernels.rs:6627-6629, 6856-6876 (for_num_elems(heads * seq)) ----------

def attention(q, k, v, head_count, head_dimension, kv_head_count=None, window_size=None, causal=False,
              key_count=None, scale=None, value_dimension=None):
    """attention_kernel, src/kernels.cu:1873-1959 (query_position_offset = kv_seq_len -
    seq_len, src/kernels.rs:6628)"""
    import torch
    q, k, v = _f32(q), _f32(k), _f32(v)
    kvh = kv_head_count or head_count
    vd = value_dimension or head_dimension
    seq = q.shape[0]
    kv_seq = key_count if key_count is not None else k.shape[0]
    out = torch.zeros(seq, head_count * vd, dtype=torch.float32, device="cuda")
    _launch("attention_kernel", _elems(head_count * seq), _THREADS,
            [_ptr(q), _ptr(k), _ptr(v), _ptr(out), _u64(seq), _u64(kv_seq), _u64(head_count), _u64(kvh),
             _u64(head_dimension), _u64(q.shape[1]), _u64(k.shape[1]), ctypes.c_int(int(causal)),
             ctypes.c_int64(-1 if window_size is None else int(window_size)), _u64(kv_seq - seq),
             ctypes.c_float(0.0 if scale is None else float(scale)), _u64(vd), _u64(v.shape[1])])
    return out
