"""GPU parity: every hot-path kernel, called through the C ABI, against the CPU oracle on the
same seeded inputs.  Bars: bit-exact for embedding gathers, add/mul/residual-add and the
half-precision ops; relative L2 <= 1e-5 for elementwise/norm/rope/softmax; <= 1e-4 for
matmul and attention."""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL_ELEMENTWISE = 1e-5
TOL_MATMUL = 1e-4


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def rng(seed=0):
    return np.random.default_rng(seed)


# ---------------------------------------------------------------------------------- elementwise
@pytest.mark.parametrize("shape", [(8, 16), (3, 5), (1000, 37), (512, 4096)])
def test_add_mul_residual_bit_exact(kernels, oracle, shape):
    r = rng(1)
    a = r.standard_normal(shape).astype(np.float32)
    b = r.standard_normal(shape).astype(np.float32)
    da, db = kernels.upload(a), kernels.upload(b)
    np.testing.assert_array_equal(kernels.download(kernels.add(da, db)), oracle.add(a, b))
    np.testing.assert_array_equal(kernels.download(kernels.mul(da, db)), oracle.mul(a, b))
    np.testing.assert_array_equal(kernels.download(kernels.residual_add(da, db)), oracle.add(a, b))


@pytest.mark.parametrize("cols,bshape", [(6, (6,)), (6, (1, 6)), (4096, (4096,)), (37, (37,))])
def test_broadcast_add_and_scalar_mul(kernels, oracle, cols, bshape):
    r = rng(2)
    a = r.standard_normal((9, cols)).astype(np.float32)
    b = r.standard_normal(bshape).astype(np.float32)
    out = kernels.download(kernels.add(kernels.upload(a), kernels.upload(b)))
    np.testing.assert_array_equal(out, oracle.add(a, b.reshape(-1)))
    s = np.array([1.75], np.float32)
    np.testing.assert_array_equal(kernels.download(kernels.mul(kernels.upload(a), kernels.upload(s))), a * s[0])


def test_shape_mismatch_is_refused(kernels, mpc):
    a = kernels.upload(np.zeros((2, 3), np.float32))
    b = kernels.upload(np.zeros((3, 2), np.float32))
    with pytest.raises(mpc.CudaError) as e:
        kernels.add(a, b)
    assert e.value.code == "ShapeUnsupported"
    with pytest.raises(mpc.CudaError) as e:
        kernels.mul(a, b)
    assert e.value.code == "ShapeUnsupported"


@pytest.mark.parametrize("n", [7, 4096, 1 << 20])
def test_silu_and_silu_mul(kernels, oracle, n):
    r = rng(3)
    g = (r.standard_normal(n) * 4).astype(np.float32)
    u = r.standard_normal(n).astype(np.float32)
    assert rel(kernels.download(kernels.silu(kernels.upload(g))), oracle.silu(g)) <= TOL_ELEMENTWISE
    assert rel(kernels.download(kernels.silu_mul(kernels.upload(g), kernels.upload(u))),
               oracle.silu_mul(g, u)) <= TOL_ELEMENTWISE


# ---------------------------------------------------------------------------------- half ops
@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("op", ["add", "mul"])
def test_half_ops_bit_exact_on_every_pattern_class(kernels, oracle, dtype, op):
    r = rng(4)
    n = 1 << 18
    a = r.integers(0, 65536, n, dtype=np.uint32).astype(np.uint16)
    b = r.integers(0, 65536, n, dtype=np.uint16 if False else np.uint32).astype(np.uint16)
    a[:65536] = np.arange(65536, dtype=np.uint16)  # every pattern once
    da, db = kernels.upload_raw(a, dtype), kernels.upload_raw(b, dtype)
    fn = kernels.add_half if op == "add" else kernels.mul_half
    got = kernels.download_raw(fn(da, db))
    exp = oracle.half_binary(a, b, dtype, op)
    bad = np.nonzero(got != exp)[0]
    assert bad.size == 0, [(hex(a[i]), hex(b[i]), hex(got[i]), hex(exp[i])) for i in bad[:8]]


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_half_ops_on_reference_fixtures(kernels, oracle, dtype):
    a = np.array([1.0, 2.5, 3.0, -4.25, 0.1, 100.0], np.float32).reshape(2, 3)
    b = np.array([6.0, 0.2, 4.0, 3.0, 0.2, -99.5], np.float32).reshape(2, 3)
    da, db = kernels.upload(a, dtype), kernels.upload(b, dtype)
    for op, fn in (("add", kernels.add_half), ("mul", kernels.mul_half)):
        got = kernels.download(fn(da, db))
        exp = oracle.half_binary_f32(a, b, dtype, op)
        np.testing.assert_array_equal(got.view(np.uint32), exp.view(np.uint32))
        got32 = kernels.download(kernels.half_binary_f32(kernels.upload(a), kernels.upload(b), dtype, op))
        np.testing.assert_array_equal(got32.view(np.uint32), exp.view(np.uint32))


def test_half_ops_refuse_mismatches(kernels, mpc):
    a = kernels.upload(np.ones(2, np.float32), "f16")
    with pytest.raises(mpc.CudaError) as e:
        kernels.add_half(a, kernels.upload(np.ones(3, np.float32), "f16"))
    assert e.value.code == "ShapeUnsupported"
    with pytest.raises(mpc.CudaError) as e:
        kernels.add_half(a, kernels.upload(np.ones(2, np.float32), "bf16"))
    assert e.value.code == "DTypeUnsupported"


def test_half_upload_download_round_trip(kernels, oracle):
    bits = np.arange(65536, dtype=np.uint16)
    for dtype in ("f16", "bf16"):
        vals = oracle.decode_half(bits, dtype)
        got = kernels.download(kernels.upload_raw(bits, dtype))
        np.testing.assert_array_equal(got.view(np.uint32), vals.view(np.uint32))
        enc = kernels.download_raw(kernels.upload(vals, dtype))
        np.testing.assert_array_equal(enc, oracle.encode_half(vals, dtype))


# ---------------------------------------------------------------------------------- embedding
@pytest.mark.parametrize("vocab,dim,n", [(32000, 512, 128), (50, 7, 33), (1000, 4096, 64)])
def test_embedding_bit_exact(kernels, oracle, vocab, dim, n):
    r = rng(5)
    table = r.standard_normal((vocab, dim)).astype(np.float32)
    ids = r.integers(0, vocab, n).astype(np.float32)
    got = kernels.download(kernels.embedding_lookup(kernels.upload(table), kernels.upload(ids)))
    exp, bad = oracle.embedding(table, ids)
    assert not bad
    np.testing.assert_array_equal(got, exp)
    got = kernels.download(kernels.embedding_lookup(kernels.upload(table), kernels.upload(ids), scale=0.5))
    np.testing.assert_array_equal(got, oracle.scale(exp, 0.5))


@pytest.mark.parametrize("bad_id", [-1.0, 1.5, 50.0, float("nan"), float("inf")])
def test_embedding_invalid_ids_fail(kernels, mpc, bad_id):
    table = kernels.upload(np.ones((50, 8), np.float32))
    with pytest.raises(mpc.CudaError) as e:
        kernels.embedding_lookup(table, kernels.upload(np.array([3.0, bad_id], np.float32)))
    assert e.value.code == "ShapeUnsupported"
    # the flag is reset: a valid lookup afterwards succeeds
    kernels.embedding_lookup(table, kernels.upload(np.array([3.0], np.float32)))


# ---------------------------------------------------------------------------------- rmsnorm
@pytest.mark.parametrize("shape", [(128, 512), (64, 4096), (7, 300), (3, 8192), (2, 20000)])
def test_rmsnorm(kernels, oracle, shape):
    r = rng(6)
    x = r.standard_normal(shape).astype(np.float32)
    w = (1 + 0.1 * r.standard_normal(shape[-1])).astype(np.float32)
    got = kernels.download(kernels.rmsnorm(kernels.upload(x), kernels.upload(w), 1e-5))
    assert rel(got, oracle.rmsnorm(x, w, 1e-5)) <= TOL_ELEMENTWISE
    got = kernels.download(kernels.rmsnorm(kernels.upload(x), None, 1e-5))
    assert rel(got, oracle.rmsnorm(x, None, 1e-5)) <= TOL_ELEMENTWISE


def test_rmsnorm_forms(kernels, oracle, mpc):
    r = rng(7)
    x = r.standard_normal((6, 256)).astype(np.float32)
    w_row = r.standard_normal((6, 256)).astype(np.float32)
    got = kernels.download(kernels.rmsnorm(kernels.upload(x), kernels.upload(w_row), 1e-6))
    assert rel(got, oracle.rmsnorm(x, w_row, 1e-6)) <= TOL_ELEMENTWISE
    w_head = r.standard_normal(64).astype(np.float32)
    got = kernels.download(kernels.rmsnorm(kernels.upload(x), kernels.upload(w_head), 1e-6, heads=(4, 64)))
    assert rel(got, oracle.rmsnorm(x, w_head, 1e-6, heads=(4, 64))) <= TOL_ELEMENTWISE
    w1 = r.standard_normal((1, 256)).astype(np.float32)
    got = kernels.download(kernels.rmsnorm(kernels.upload(x), kernels.upload(w1), 1e-6))
    assert rel(got, oracle.rmsnorm(x, w1.reshape(-1), 1e-6)) <= TOL_ELEMENTWISE
    with pytest.raises(mpc.CudaError):
        kernels.rmsnorm(kernels.upload(x), kernels.upload(w_head), 0.0)
    with pytest.raises(mpc.CudaError):
        kernels.rmsnorm(kernels.upload(x), kernels.upload(w_head), 1e-6, heads=(3, 64))


# ---------------------------------------------------------------------------------- rope
ROPE_CASES = [
    dict(shape=(128, 512), head_count=8, dimension=64, base=10000.0),
    dict(shape=(256, 4096), head_count=32, dimension=128, base=500000.0),
    dict(shape=(64, 512), head_count=8, dimension=64, base=10000.0, pairing="half_split", position_offset=1000),
    dict(shape=(3, 12), head_count=2, dimension=4, base=10000.0),
    dict(shape=(3, 12), head_count=2, dimension=4, base=10000.0, pairing="half_split"),
    dict(shape=(40, 256), head_count=2, dimension=96, base=10000.0, rotated_pairs=20),
    dict(shape=(40, 256), head_count=4, dimension=64, base=500000.0, banded=(8.0, 1.0, 4.0, 8192.0)),
    dict(shape=(40, 256), head_count=4, dimension=64, base=10000.0, yarn=(4.0, 3.0, 20.0, 1.1)),
    dict(shape=(5, 30), head_count=3, dimension=6, base=100.0, scale=0.5),
]


@pytest.mark.parametrize("case", ROPE_CASES)
def test_rope(kernels, oracle, case):
    c = dict(case)
    shape = c.pop("shape")
    pairing = c.pop("pairing", "interleaved")
    x = rng(8).standard_normal(shape).astype(np.float32)
    got = kernels.download(kernels.rope(kernels.upload(x), pairing=pairing, **c))
    exp = oracle.rope(x, half_split=pairing == "half_split", **c)
    assert rel(got, exp) <= TOL_ELEMENTWISE


def test_rope_validation(kernels, mpc):
    x = kernels.upload(np.zeros((4, 12), np.float32))
    for kw in (dict(head_count=5, dimension=2), dict(head_count=2, dimension=3), dict(head_count=2, dimension=8),
               dict(head_count=2, dimension=4, base=-1.0)):
        with pytest.raises(mpc.CudaError) as e:
            kernels.rope(x, **kw)
        assert e.value.code == "ShapeUnsupported"


# ---------------------------------------------------------------------------------- softmax
@pytest.mark.parametrize("shape", [(1000, 2048), (64, 100), (33, 513), (16, 5000), (4096, 128)])
def test_softmax(kernels, oracle, shape):
    x = (rng(9).standard_normal(shape) * 2).astype(np.float32)
    got = kernels.download(kernels.softmax_rows(kernels.upload(x)))
    exp, flag = oracle.softmax(x)
    assert not flag
    assert rel(got, exp) <= TOL_ELEMENTWISE


def test_softmax_non_finite_row_fails(kernels, mpc):
    x = np.zeros((4, 64), np.float32)
    x[2] = -np.inf
    with pytest.raises(mpc.CudaError) as e:
        kernels.softmax_rows(kernels.upload(x))
    assert e.value.code == "ExecutionFailed"
    x[2] = 0
    kernels.softmax_rows(kernels.upload(x))


# ---------------------------------------------------------------------------------- matmul
MATMUL_SHAPES = [
    (1, 4096, 512), (1, 1000, 70), (3, 129, 64), (16, 4096, 4096), (4, 50, 40),
    (17, 64, 96), (128, 512, 512), (128, 512, 1376), (128, 1376, 512), (200, 904, 136),
    (256, 1024, 768), (300, 129, 65), (513, 257, 130),
    # split k with many k-blocks per CTA (partials received in the drained ring): 128- and
    # 32-wide tiles; and the 32-wide tile with its own receive region
    (128, 4096, 512), (128, 2048, 2048), (64, 4096, 32), (64, 512, 32),
    # GEMV: the most k splits of one cluster, a long k, and k not a multiple of 4 (TMA-staged
    # path); transposed A with a long k takes the two-kernel path (test_matmul_transposed)
    (8, 16384, 256), (16, 40000, 128), (5, 4098, 260),
    # GEMV item path (m <= 4): two and three rows, a ragged last column tile, k shorter than one
    # item, and a long k (many items per column tile summed by the last one)
    (2, 4096, 4096), (3, 8192, 200), (4, 1024, 1000), (1, 36, 64), (1, 65536, 96),
]


@pytest.mark.parametrize("m,k,n", MATMUL_SHAPES)
def test_matmul(kernels, oracle, m, k, n):
    r = rng(10)
    a = (r.standard_normal((m, k)) / math.sqrt(k)).astype(np.float32)
    b = (r.standard_normal((k, n))).astype(np.float32)
    got = kernels.download(kernels.matmul(kernels.upload(a), kernels.upload(b)))
    assert rel(got, oracle.matmul(a, b)) <= TOL_MATMUL


@pytest.mark.parametrize("m,k,n", [(128, 512, 512), (200, 904, 136), (128, 2048, 2048), (513, 257, 132),
                                   (64, 4096, 32), (300, 129, 65), (1, 4096, 512), (3, 2048, 1000),
                                   (16, 4096, 256)])
def test_matmul_with_weight_b(kernels, oracle, m, k, n):
    # B marked as a weight: its tensor-core operand form is built by the first call and kept;
    # both calls match the oracle and each other.  (Plain B at M <= 128 is split inside the
    # kernel: the other matmul tests.)
    r = rng(15)
    a = (r.standard_normal((m, k)) / math.sqrt(k)).astype(np.float32)
    b = r.standard_normal((k, n)).astype(np.float32)
    da, db = kernels.upload(a), kernels.upload(b).set_weight()
    first = kernels.download(kernels.matmul(da, db))
    second = kernels.download(kernels.matmul(da, db))
    assert rel(first, oracle.matmul(a, b)) <= TOL_MATMUL
    np.testing.assert_array_equal(first, second)


def test_gemv_weight_written_by_the_preceding_kernel(kernels, oracle):
    # A buffer that a kernel has just written and that then becomes a weight: the next matmul
    # must wait for that kernel before reading it; later matmuls may read it early.
    r = rng(16)
    a = (r.standard_normal((2, 2048)) / math.sqrt(2048)).astype(np.float32)
    x = r.standard_normal((2048, 768)).astype(np.float32)
    y = r.standard_normal((2048, 768)).astype(np.float32)
    da = kernels.upload(a)
    for _ in range(3):
        w = kernels.add(kernels.upload(x), kernels.upload(y)).set_weight()
        first = kernels.download(kernels.matmul(da, w))
        second = kernels.download(kernels.matmul(da, w))
        exp = oracle.matmul(a, x + y)
        assert rel(first, exp) <= TOL_MATMUL
        np.testing.assert_array_equal(first, second)


@pytest.mark.parametrize("m,k,n", [(1, 300, 70), (16, 256, 128), (130, 200, 96), (16, 40000, 128)])
@pytest.mark.parametrize("ta,tb", [(True, False), (False, True), (True, True)])
def test_matmul_transposed(kernels, oracle, m, k, n, ta, tb):
    r = rng(11)
    a = r.standard_normal((k, m) if ta else (m, k)).astype(np.float32)
    b = r.standard_normal((n, k) if tb else (k, n)).astype(np.float32)
    got = kernels.download(kernels.matmul(kernels.upload(a), kernels.upload(b), ta, tb))
    assert rel(got, oracle.matmul(a, b, ta, tb)) <= TOL_MATMUL


@pytest.mark.parametrize("m,k", [(1, 256), (16, 256), (128, 256), (300, 256), (128, 4096), (3, 4096)])
def test_matmul_bias_and_residual(kernels, oracle, m, k):
    r = rng(12)
    n = 192
    a = r.standard_normal((m, k)).astype(np.float32)
    b = r.standard_normal((k, n)).astype(np.float32)
    bias = r.standard_normal(n).astype(np.float32)
    res = r.standard_normal((m, n)).astype(np.float32)
    da, db = kernels.upload(a), kernels.upload(b)
    got = kernels.download(kernels.matmul_bias(da, db, kernels.upload(bias)))
    assert rel(got, oracle.matmul(a, b, addend=bias, addend_mode=1)) <= TOL_MATMUL
    got = kernels.download(kernels.matmul_residual(da, db, kernels.upload(res)))
    assert rel(got, oracle.matmul(a, b, addend=res, addend_mode=2)) <= TOL_MATMUL


@pytest.mark.parametrize("m,k,n", [(1, 512, 1376), (16, 512, 256), (128, 512, 1376), (200, 300, 136),
                                   (128, 4096, 256), (4, 4096, 1000)])
def test_gated_matmul(kernels, oracle, m, k, n):
    r = rng(13)
    a = r.standard_normal((m, k)).astype(np.float32)
    g = (r.standard_normal((k, n)) * 0.05).astype(np.float32)
    u = (r.standard_normal((k, n)) * 0.05).astype(np.float32)
    got = kernels.download(kernels.gated_matmul(kernels.upload(a), kernels.upload(g), kernels.upload(u)))
    assert rel(got, oracle.gated_matmul(a, g, u)) <= TOL_MATMUL


# The few-row tensor-core path (8 <= M <= 16, k and n multiples of 4): the weight as the MMA's
# 128-row operand, raw tiles split into tf32 hi / lo in the kernel, k split across a cluster.
FEWROW_TC_SHAPES = [(8, 4096, 4096), (11, 4096, 4096), (16, 4096, 4096), (16, 4100, 260), (9, 64, 4),
                    (16, 32, 128), (12, 12288, 136), (16, 1376, 512), (10, 512, 1376), (16, 256, 65536)]


@pytest.mark.parametrize("m,k,n", FEWROW_TC_SHAPES)
@pytest.mark.parametrize("weight", [False, True])
def test_fewrow_tensor_core_matmul(kernels, oracle, m, k, n, weight):
    r = rng(17)
    a = (r.standard_normal((m, k)) / math.sqrt(k)).astype(np.float32)
    b = r.standard_normal((k, n)).astype(np.float32)
    db = kernels.upload(b)
    if weight:
        db.set_weight()
    da = kernels.upload(a)
    first = kernels.download(kernels.matmul(da, db))
    assert rel(first, oracle.matmul(a, b)) <= TOL_MATMUL
    np.testing.assert_array_equal(first, kernels.download(kernels.matmul(da, db)))  # deterministic


_FEWROW_TC_CHILD = r"""
import importlib, json, math, sys
import numpy as np
sys.path.insert(0, sys.argv[1])
mpc = importlib.import_module("magnetar-provider-cuda_b200")
kernels = mpc.CudaKernels(0)
r = np.random.default_rng(23)
out = []
for m, k, n, gated in [(16, 4096, 4096, 0), (9, 64, 4, 0), (12, 4100, 260, 0), (10, 512, 1376, 1), (16, 1376, 512, 0)]:
    a = (r.standard_normal((m, k)) / math.sqrt(k)).astype(np.float32)
    b = r.standard_normal((k, n)).astype(np.float32)
    da, db = kernels.upload(a), kernels.upload(b)
    if gated:
        u = r.standard_normal((k, n)).astype(np.float32)
        got = kernels.download(kernels.gated_matmul(da, db, kernels.upload(u))).astype(np.float64)
        g = a.astype(np.float64) @ b.astype(np.float64)
        exp = g / (1.0 + np.exp(-g)) * (a.astype(np.float64) @ u.astype(np.float64))
    else:
        db.set_weight()
        got = kernels.download(kernels.matmul(da, db)).astype(np.float64)
        exp = a.astype(np.float64) @ b.astype(np.float64)
    out.append(float(np.linalg.norm(got - exp) / np.linalg.norm(exp)))
kernels.close()
print(json.dumps(out))
"""


def test_fewrow_tensor_core_form_in_a_fresh_process():
    # The f32 tensor-core few-row form is off by default and chosen once per process
    # (MAGNETAR_CUDA_FEWROW_TC): a child process with it on checks it against f64 products.
    import json
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, MAGNETAR_CUDA_FEWROW_TC="2")
    res = subprocess.run([sys.executable, "-c", _FEWROW_TC_CHILD, root], env=env, capture_output=True, text=True,
                         timeout=300)
    assert res.returncode == 0, res.stderr[-2000:]
    errs = json.loads(res.stdout.strip().splitlines()[-1])
    assert len(errs) == 5 and max(errs) <= TOL_MATMUL, errs


_SWITCHED_PATHS_CHILD = r"""
import importlib, json, math, sys
import numpy as np
sys.path.insert(0, sys.argv[1])
mpc = importlib.import_module("magnetar-provider-cuda_b200")
from oracle import oracle as orc
orc.build()
kernels = mpc.CudaKernels(0)
r = np.random.default_rng(29)
out = []
for seq, heads, kvh, d, causal in [(640, 2, 2, 128, True), (384, 4, 2, 64, False), (300, 2, 1, 128, True)]:
    q = r.standard_normal((seq, heads * d)).astype(np.float32)
    k = r.standard_normal((seq, kvh * d)).astype(np.float32)
    v = r.standard_normal((seq, kvh * d)).astype(np.float32)
    got = kernels.download(kernels.attention(kernels.upload(q), kernels.upload(k), kernels.upload(v), heads, d,
                                             kv_head_count=kvh, causal=causal))
    exp = orc.attention(q, k, v, heads, d, kv_head_count=kvh, causal=causal)
    out.append(float(np.linalg.norm(got - exp) / np.linalg.norm(exp)))
for m, kk, n in [(128, 512, 1376), (64, 1376, 512)]:
    a = r.standard_normal((m, kk)).astype(np.float32)
    g = (r.standard_normal((kk, n)) * 0.05).astype(np.float32)
    u = (r.standard_normal((kk, n)) * 0.05).astype(np.float32)
    dg, du = kernels.upload(g), kernels.upload(u)
    dg.set_weight()
    du.set_weight()
    got = kernels.download(kernels.gated_matmul(kernels.upload(a), dg, du))
    exp = orc.gated_matmul(a, g, u)
    out.append(float(np.linalg.norm(got - exp) / np.linalg.norm(exp)))
kernels.close()
print(json.dumps(out))
"""


@pytest.mark.parametrize("env", [{"MAGNETAR_CUDA_ATTN_ONE_TILE": "1"}, {"MAGNETAR_CUDA_GEMM_RAW_WEIGHTS": "0"},
                                 {"MAGNETAR_CUDA_GEMM_RAW_WEIGHTS": "1"}])
def test_switched_paths_in_a_fresh_process(env):
    # Paths chosen once per process by a switch: the one-query-tile attention kernel (with its Q
    # split pass) and the GEMM's weight form forced prepared or raw at every k, against the oracle.
    import json
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    res = subprocess.run([sys.executable, "-c", _SWITCHED_PATHS_CHILD, root], env=dict(os.environ, **env),
                         capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    errs = json.loads(res.stdout.strip().splitlines()[-1])
    assert len(errs) == 5 and max(errs) <= TOL_MATMUL, errs


@pytest.mark.parametrize("m,k,n", [(16, 2048, 1000), (8, 512, 1376), (13, 4096, 128)])
def test_fewrow_tensor_core_epilogues(kernels, oracle, m, k, n):
    r = rng(18)
    a = r.standard_normal((m, k)).astype(np.float32)
    g = (r.standard_normal((k, n)) * 0.05).astype(np.float32)
    u = (r.standard_normal((k, n)) * 0.05).astype(np.float32)
    bias = r.standard_normal(n).astype(np.float32)
    res = r.standard_normal((m, n)).astype(np.float32)
    da, dg, du = kernels.upload(a), kernels.upload(g), kernels.upload(u)
    assert rel(kernels.download(kernels.gated_matmul(da, dg, du)), oracle.gated_matmul(a, g, u)) <= TOL_MATMUL
    got = kernels.download(kernels.matmul_bias(da, dg, kernels.upload(bias)))
    assert rel(got, oracle.matmul(a, g, addend=bias, addend_mode=1)) <= TOL_MATMUL
    got = kernels.download(kernels.matmul_residual(da, dg, kernels.upload(res)))
    assert rel(got, oracle.matmul(a, g, addend=res, addend_mode=2)) <= TOL_MATMUL


def test_fewrow_tensor_core_keeps_f32_activation_precision(kernels):
    # src/tests_conformance.rs:807-846 at 16 rows: 1 + 2^-12 activations survive the tf32 split.
    m, k, n = 16, 900, 132
    a = np.full((m, k), 1.0 + 2.0 ** -12, np.float32)
    w = np.abs(rng(21).standard_normal((k, n)).astype(np.float32))
    w = (w.view(np.uint32) & 0xFFFF0000).view(np.float32)
    got = kernels.download(kernels.matmul(kernels.upload(a), kernels.upload(w))).astype(np.float64)
    exp = a.astype(np.float64) @ w.astype(np.float64)
    assert rel(got, exp) <= 1e-6


@pytest.mark.parametrize("m,k,n", [(70, 900, 130), (200, 904, 136)])
def test_matmul_keeps_f32_activation_precision(kernels, m, k, n):
    # src/tests_conformance.rs:807-846
    a = np.full((m, k), 1.0 + 2.0 ** -12, np.float32)
    w = np.abs(rng(21).standard_normal((k, n)).astype(np.float32))
    w = (w.view(np.uint32) & 0xFFFF0000).view(np.float32)
    got = kernels.download(kernels.matmul(kernels.upload(a), kernels.upload(w))).astype(np.float64)
    exp = (1.0 + 2.0 ** -12) * w.astype(np.float64).sum(axis=0)
    assert np.all(np.abs(got - exp) <= 5e-5 * exp)


def test_matmul_near_f32_max_stays_finite(kernels):
    # src/tests_conformance.rs:852-880
    m, k, n = 64, 256, 256
    a = np.full((m, k), np.finfo(np.float32).max, np.float32)
    b = np.full((k, n), 2.0 ** -120, np.float32)
    got = kernels.download(kernels.matmul(kernels.upload(a), kernels.upload(b)))
    exp = float(np.finfo(np.float32).max) * 2.0 ** -120 * k
    assert np.all(np.isfinite(got)) and np.all(np.abs(got / exp - 1) < 1e-4)


def test_matmul_shape_errors(kernels, mpc):
    a = kernels.upload(np.zeros((4, 5), np.float32))
    with pytest.raises(mpc.CudaError) as e:
        kernels.matmul(a, kernels.upload(np.zeros((4, 5), np.float32)))
    assert e.value.code == "ShapeUnsupported"
    with pytest.raises(mpc.CudaError) as e:
        kernels.matmul(kernels.upload(np.zeros(5, np.float32)), a)
    assert e.value.code == "ShapeUnsupported"
    with pytest.raises(mpc.CudaError) as e:
        kernels.matmul_bias(a, kernels.upload(np.zeros((5, 3), np.float32)), kernels.upload(np.zeros(4, np.float32)))
    assert e.value.code == "ShapeUnsupported"


# ---------------------------------------------------------------------------------- attention
ATTN_CASES = [
    dict(seq=128, kv=128, heads=8, kvh=8, d=64, causal=True),
    dict(seq=200, kv=200, heads=4, kvh=4, d=128, causal=True),
    dict(seq=70, kv=70, heads=4, kvh=2, d=64, causal=True),
    dict(seq=33, kv=33, heads=2, kvh=2, d=64, causal=False),
    dict(seq=64, kv=64, heads=4, kvh=1, d=64, causal=True, window=16),
    dict(seq=20, kv=100, heads=2, kvh=2, d=128, causal=True),
    dict(seq=20, kv=100, heads=2, kvh=2, d=64, causal=True, key_count=60),
    dict(seq=40, kv=40, heads=2, kvh=2, d=64, causal=True, scale=0.3),
    dict(seq=37, kv=37, heads=3, kvh=3, d=48, causal=True),
    dict(seq=30, kv=30, heads=2, kvh=2, d=64, causal=True, vd=32),
    dict(seq=1, kv=300, heads=4, kvh=2, d=64, causal=True),
    dict(seq=3, kv=3, heads=1, kvh=1, d=2, causal=True),
    dict(seq=640, kv=640, heads=2, kvh=2, d=128, causal=True),
    dict(seq=384, kv=512, heads=4, kvh=2, d=64, causal=False),
    dict(seq=300, kv=300, heads=2, kvh=1, d=128, causal=True, window=100),
    dict(seq=129, kv=1000, heads=2, kvh=2, d=64, causal=True, key_count=777),
    # spans too long for the short (span-resident) kernel: tensor-core path with a window,
    # GQA with a query offset, non-causal
    dict(seq=300, kv=300, heads=2, kvh=1, d=128, causal=True, window=250),
    dict(seq=70, kv=420, heads=4, kvh=2, d=64, causal=True),
    dict(seq=33, kv=400, heads=2, kvh=2, d=64, causal=False),
    # short kernel: a window over a long sequence, the 384-key capacity, D = 32, D = 128
    dict(seq=50, kv=300, heads=3, kvh=1, d=64, causal=True, window=40),
    dict(seq=16, kv=384, heads=2, kvh=2, d=64, causal=True),
    dict(seq=100, kv=100, heads=2, kvh=2, d=32, causal=True),
    dict(seq=129, kv=129, heads=2, kvh=2, d=128, causal=False),
    # one query row (decode): keys split across CTAs in chunks of 128 -- one chunk, a ragged
    # last chunk, many chunks with GQA, a window, a key count, non-causal, D = 256, Dv != D,
    # a head dimension that is no multiple of 4
    dict(seq=1, kv=1, heads=2, kvh=2, d=64, causal=True),
    dict(seq=1, kv=129, heads=4, kvh=4, d=128, causal=True),
    dict(seq=1, kv=4096, heads=32, kvh=8, d=128, causal=True),
    dict(seq=1, kv=1000, heads=4, kvh=2, d=64, causal=True, window=300),
    dict(seq=1, kv=1000, heads=4, kvh=2, d=64, causal=True, key_count=513),
    dict(seq=1, kv=700, heads=2, kvh=2, d=64, causal=False),
    dict(seq=1, kv=300, heads=2, kvh=1, d=256, causal=True),
    dict(seq=1, kv=300, heads=2, kvh=2, d=64, causal=True, vd=96),
    dict(seq=1, kv=200, heads=3, kvh=3, d=30, causal=True),
]


@pytest.mark.parametrize("c", ATTN_CASES)
def test_attention(kernels, oracle, c):
    r = rng(14)
    vd = c.get("vd", c["d"])
    q = r.standard_normal((c["seq"], c["heads"] * c["d"])).astype(np.float32)
    k = r.standard_normal((c["kv"], c["kvh"] * c["d"])).astype(np.float32)
    v = r.standard_normal((c["kv"], c["kvh"] * vd)).astype(np.float32)
    kw = dict(kv_head_count=c["kvh"], window_size=c.get("window"), causal=c["causal"],
              key_count=c.get("key_count"), scale=c.get("scale"), value_dimension=c.get("vd"))
    got = kernels.download(kernels.attention(kernels.upload(q), kernels.upload(k), kernels.upload(v),
                                             c["heads"], c["d"], **kw))
    exp = oracle.attention(q, k, v, c["heads"], c["d"], **kw)
    assert rel(got, exp) <= TOL_MATMUL


def test_kv_write(kernels, mpc):
    # src/kernels.rs:2278-2325: rows over the store's rows row_offset.. in place, the rest kept
    r = rng(17)
    store = r.standard_normal((64, 96)).astype(np.float32)
    rows = r.standard_normal((5, 96)).astype(np.float32)
    ds = kernels.upload(store)
    kernels.kv_write(ds, kernels.upload(rows), 40)
    exp = store.copy()
    exp[40:45] = rows
    np.testing.assert_array_equal(kernels.download(ds), exp)
    kernels.kv_write(ds, kernels.upload(rows[:1]), 63)  # the last row
    exp[63] = rows[0]
    np.testing.assert_array_equal(kernels.download(ds), exp)
    odd = r.standard_normal((3, 7)).astype(np.float32)  # unvectorised width
    do = kernels.upload(np.zeros((9, 7), np.float32))
    kernels.kv_write(do, kernels.upload(odd), 2)
    np.testing.assert_array_equal(kernels.download(do)[2:5], odd)
    with pytest.raises(mpc.CudaError) as e:
        kernels.kv_write(ds, kernels.upload(rows), 60)  # past the store's rows
    assert e.value.code == "ShapeUnsupported"
    with pytest.raises(mpc.CudaError) as e:
        kernels.kv_write(ds, kernels.upload(np.zeros((2, 95), np.float32)), 0)
    assert e.value.code == "ShapeUnsupported"
    np.testing.assert_array_equal(kernels.download(ds), exp)  # failed writes changed nothing


def test_attention_large_values_stay_finite(kernels):
    # src/tests_conformance.rs:884-914
    rows = 70
    q = np.zeros((rows, 64), np.float32)
    v = np.full((rows, 64), 1e38, np.float32)
    got = kernels.download(kernels.attention(kernels.upload(q), kernels.upload(q), kernels.upload(v), 1, 64,
                                             causal=True))
    assert np.all(np.isfinite(got)) and np.all(np.abs(got / 1e38 - 1) < 1e-4)


@pytest.mark.parametrize("d", [64, 128])
def test_tensor_core_attention_large_values_keep_the_weighted_mean_form(kernels, oracle, d):
    # src/tests_conformance.rs:884-914 at a length the tensor-core kernel takes: |V| near f32::MAX
    # would overflow an unnormalised sum, so the kernel keeps the output a weighted mean of V rows.
    rows = 640
    q = np.zeros((rows, d), np.float32)
    v = np.full((rows, d), 1e38, np.float32)
    got = kernels.download(kernels.attention(kernels.upload(q), kernels.upload(q), kernels.upload(v), 1, d,
                                             causal=True))
    assert np.all(np.isfinite(got)) and np.all(np.abs(got / 1e38 - 1) < 1e-4)
    # large but distinct values: the weighted-mean form against the oracle
    r = rng(31)
    q = r.standard_normal((rows, 2 * d)).astype(np.float32)
    k = r.standard_normal((rows, 2 * d)).astype(np.float32)
    v = (r.standard_normal((rows, 2 * d)) * 1e30).astype(np.float32)
    got = kernels.download(kernels.attention(kernels.upload(q), kernels.upload(k), kernels.upload(v), 2, d,
                                             causal=True))
    assert rel(got, oracle.attention(q, k, v, 2, d, causal=True)) <= TOL_MATMUL


@pytest.mark.parametrize("causal", [True, False])
def test_tensor_core_attention_rescales_when_the_row_max_jumps(kernels, oracle, causal):
    # Scores that grow along the keys by far more than 2^12 in log2 units from one 64-key tile to
    # the next: the kernel's reference max has to move (and the output be rescaled) many times.
    rows, d = 700, 128
    r = rng(32)
    q = r.standard_normal((rows, d)).astype(np.float32)
    k = r.standard_normal((rows, d)).astype(np.float32)
    k *= (1.0 + np.arange(rows, dtype=np.float32) / 16.0)[:, None]
    v = r.standard_normal((rows, d)).astype(np.float32)
    got = kernels.download(kernels.attention(kernels.upload(q), kernels.upload(k), kernels.upload(v), 1, d,
                                             causal=causal))
    assert rel(got, oracle.attention(q, k, v, 1, d, causal=causal)) <= TOL_MATMUL


@pytest.mark.parametrize("m,k,n", [(128, 512, 1376), (96, 2048, 256), (128, 2049, 136), (40, 1376, 512)])
def test_weights_read_raw_or_prepared(kernels, oracle, m, k, n):
    # Weights are read raw (split in the GEMM) up to k = 2048 and through their prepared hi / lo
    # form beyond: plain, gated and residual forms on both sides of the switch.
    r = rng(33)
    a = r.standard_normal((m, k)).astype(np.float32)
    g = (r.standard_normal((k, n)) * 0.05).astype(np.float32)
    u = (r.standard_normal((k, n)) * 0.05).astype(np.float32)
    res = r.standard_normal((m, n)).astype(np.float32)
    da, dg, du = kernels.upload(a), kernels.upload(g), kernels.upload(u)
    dg.set_weight()
    du.set_weight()
    for _ in range(2):  # the first call builds the prepared forms, the second reads them settled
        assert rel(kernels.download(kernels.matmul(da, dg)), oracle.matmul(a, g)) <= TOL_MATMUL
        got = kernels.download(kernels.gated_matmul(da, dg, du))
        assert rel(got, oracle.gated_matmul(a, g, u)) <= TOL_MATMUL
        got = kernels.download(kernels.matmul_residual(da, dg, kernels.upload(res)))
        assert rel(got, oracle.matmul(a, g, addend=res, addend_mode=2)) <= TOL_MATMUL


def test_attention_validation(kernels, mpc):
    q = kernels.upload(np.zeros((4, 8), np.float32))
    for kw in (dict(head_count=3, head_dimension=4), dict(head_count=2, head_dimension=4, kv_head_count=3),
               dict(head_count=2, head_dimension=4, window_size=0, causal=True),
               dict(head_count=2, head_dimension=4, window_size=2, causal=False),
               dict(head_count=2, head_dimension=4, key_count=9),
               dict(head_count=2, head_dimension=4, scale=-1.0)):
        with pytest.raises(mpc.CudaError) as e:
            kernels.attention(q, q, q, **kw)
        assert e.value.code == "ShapeUnsupported", kw


# ---------------------------------------------------------------------------------- full-size properties
def test_full_size_memory_bound_suite_properties(kernels, oracle):
    """Config 4 sizes: [8192, 4096] through add (bit-exact vs numpy), rmsnorm rows have unit
    RMS before the gain, softmax rows sum to one."""
    r = rng(15)
    x = r.standard_normal((8192, 4096)).astype(np.float32)
    y = r.standard_normal((8192, 4096)).astype(np.float32)
    dx, dy = kernels.upload(x), kernels.upload(y)
    np.testing.assert_array_equal(kernels.download(kernels.add(dx, dy)), x + y)
    n = kernels.download(kernels.rmsnorm(dx, None, 1e-5))
    rms = np.sqrt((n.astype(np.float64) ** 2).mean(axis=1))
    assert np.all(np.abs(rms - 1) < 1e-4)
    s = kernels.download(kernels.softmax_rows(kernels.upload(x[:2048, :2048] * 2)))
    assert np.all(np.abs(s.astype(np.float64).sum(axis=1) - 1) < 1e-5)


def test_gemm_sweep_full_size_linearity(kernels):
    """Config 2 size (M=2048, N=K=4096): A(B1 + B2) == A B1 + A B2 within the matmul bar."""
    r = rng(16)
    k = 4096
    a = (r.standard_normal((2048, k)) / math.sqrt(k)).astype(np.float32)
    b1 = (r.standard_normal((k, k)) / math.sqrt(k)).astype(np.float32)
    b2 = (r.standard_normal((k, k)) / math.sqrt(k)).astype(np.float32)
    da = kernels.upload(a)
    lhs = kernels.download(kernels.matmul(da, kernels.upload(b1 + b2)))
    rhs = kernels.download(kernels.add(kernels.matmul(da, kernels.upload(b1)), kernels.matmul(da, kernels.upload(b2))))
    assert rel(lhs, rhs) <= TOL_MATMUL
    # and a row sample against float64
    exp = a[:8].astype(np.float64) @ (b1 + b2).astype(np.float64)
    assert rel(lhs[:8], exp) <= TOL_MATMUL


def test_buffers_outlive_a_closed_device(mpc):
    # A buffer released after its device handle was closed frees into the still-live pool,
    # and the closed handle refuses new work with DeviceUnavailable instead of crashing.
    import ctypes
    import importlib
    N = importlib.import_module("magnetar-provider-cuda_b200._native")
    unavailable = [c for c, name in N.STATUS_NAMES.items() if name == "DeviceUnavailable"][0]
    k = mpc.CudaKernels(0)
    a = k.upload(np.ones((4, 4), np.float32))
    b = k.add(a, a)
    stale = ctypes.c_void_p(k.handle.value)
    k.close()
    out = ctypes.c_void_p()
    assert N.lib().mg_add(stale, a.handle, b.handle, ctypes.byref(out)) == unavailable
    a.release()
    b.release()  # the last reference: the device goes now


def test_layered_elementwise_forms(kernels, oracle, mpc):
    # gelu (tanh), sigmoid, softcap and row-scale against the oracle (src/tests_conformance.rs:
    # 4717-4732, 4945-4990); vectorised and ragged sizes
    r = rng(18)
    for shape in ((3, 70), (64, 1024), (5, 7)):
        x = (r.standard_normal(shape) * 4).astype(np.float32)
        dx = kernels.upload(x)
        assert rel(kernels.download(kernels.gelu_tanh(dx)), oracle.gelu_tanh(x)) <= TOL_ELEMENTWISE
        assert rel(kernels.download(kernels.sigmoid(dx)), oracle.sigmoid(x)) <= TOL_ELEMENTWISE
        assert rel(kernels.download(kernels.softcap(dx, 1.5)), oracle.softcap(x, 1.5)) <= TOL_ELEMENTWISE
        s = r.standard_normal(shape[0]).astype(np.float32)
        for sd in (kernels.upload(s), kernels.upload(s.reshape(-1, 1))):
            np.testing.assert_array_equal(kernels.download(kernels.row_scale(dx, sd)), oracle.row_scale(x, s))
    with pytest.raises(mpc.CudaError) as e:
        kernels.softcap(dx, 0.0)
    assert e.value.code == "ShapeUnsupported"
    with pytest.raises(mpc.CudaError) as e:
        kernels.row_scale(dx, kernels.upload(np.ones(6, np.float32)))
    assert e.value.code == "ShapeUnsupported"


def test_concat_rows_and_heads(kernels, oracle, mpc):
    # src/kernels.rs:3058-3100, 7084-7130; src/tests_conformance.rs:5606-5640
    r = rng(19)
    a = r.standard_normal((3, 4, 5)).astype(np.float32)
    b = r.standard_normal((2, 4, 5)).astype(np.float32)
    got = kernels.concat(kernels.upload(a), kernels.upload(b))
    assert got.shape == (5, 4, 5)
    np.testing.assert_array_equal(kernels.download(got), oracle.concat(a, b))
    with pytest.raises(mpc.CudaError) as e:
        kernels.concat(kernels.upload(a), kernels.upload(np.zeros((2, 4, 6), np.float32)))
    assert e.value.code == "ShapeUnsupported"
    for heads, aw, second, bw in ((4, 6, 4, 2), (16, 128, 1, 64), (3, 5, 3, 3), (2, 8, 1, 4)):
        x = r.standard_normal((5, heads * aw)).astype(np.float32)
        y = r.standard_normal((5, second * bw)).astype(np.float32)
        got = kernels.concat_heads(kernels.upload(x), kernels.upload(y), heads, second)
        np.testing.assert_array_equal(kernels.download(got), oracle.concat_heads(x, y, heads, second))
    x = kernels.upload(r.standard_normal((5, 12)).astype(np.float32))
    for y, second in ((np.zeros((4, 3), np.float32), 1), (np.zeros((5, 6), np.float32), 2)):
        with pytest.raises(mpc.CudaError) as e:
            kernels.concat_heads(x, kernels.upload(y), 4, second)
        assert e.value.code == "ShapeUnsupported"


@pytest.mark.parametrize("rows,groups,k,n", [(3, 2, 8, 5), (16, 4, 64, 32), (1, 8, 128, 96), (7, 3, 33, 17)])
@pytest.mark.parametrize("tb", [False, True])
def test_batched_matmul(kernels, oracle, rows, groups, k, n, tb):
    r = rng(20)
    a = r.standard_normal((rows, groups * k)).astype(np.float32)
    b = r.standard_normal((groups * n, k) if tb else (groups * k, n)).astype(np.float32)
    got = kernels.download(kernels.batched_matmul(kernels.upload(a), kernels.upload(b), groups, tb))
    assert rel(got, oracle.batched_matmul(a, b, groups, tb)) <= TOL_MATMUL


def test_batched_matmul_shape_errors(kernels, mpc):
    a = kernels.upload(np.zeros((2, 12), np.float32))
    for b, groups, tb in ((np.zeros((12, 4), np.float32), 5, False), (np.zeros((10, 4), np.float32), 2, False),
                          (np.zeros((6, 5), np.float32), 2, True)):
        with pytest.raises(mpc.CudaError) as e:
            kernels.batched_matmul(a, kernels.upload(b), groups, tb)
        assert e.value.code == "ShapeUnsupported"


def _bf16_exact(x):
    return (np.asarray(x, np.float32).view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32)


@pytest.mark.parametrize("m,k,n", [(256, 512, 384), (200, 904, 136), (2048, 256, 256), (128, 1024, 512)])
def test_matmul_with_an_exact_weight_drops_its_lo_term(kernels, oracle, m, k, n):
    # A weight whose values are exactly bfloat16 (so tf32): its prepared lo term is zero and the
    # matmul reads and multiplies hi alone -- bit-identical to multiplying the zero term as well
    # (the per-call split of the same values, which keeps all three products), and to the oracle
    # within the matmul tolerance.
    r = rng(22)
    a = (r.standard_normal((m, k)) / math.sqrt(k)).astype(np.float32)
    b = _bf16_exact(r.standard_normal((k, n)))
    da = kernels.upload(a)
    db = kernels.upload(b).set_weight()
    first = kernels.download(kernels.matmul(da, db))
    second = kernels.download(kernels.matmul(da, db))
    assert rel(first, oracle.matmul(a, b)) <= TOL_MATMUL
    np.testing.assert_array_equal(first, second)
    if m > 128:  # the per-call form goes through the same kernel (B split into a scratch form)
        np.testing.assert_array_equal(second, kernels.download(kernels.matmul(da, kernels.upload(b))))


@pytest.mark.parametrize("exact_up", [True, False])
def test_gated_matmul_with_exact_weights(kernels, oracle, exact_up):
    r = rng(23)
    m, k, n = 256, 512, 320
    a = r.standard_normal((m, k)).astype(np.float32)
    g = _bf16_exact(r.standard_normal((k, n)) * 0.05)
    u = (r.standard_normal((k, n)) * 0.05).astype(np.float32)
    if exact_up:
        u = _bf16_exact(u)
    da, dg, du = kernels.upload(a), kernels.upload(g).set_weight(), kernels.upload(u).set_weight()
    got = kernels.download(kernels.gated_matmul(da, dg, du))
    got2 = kernels.download(kernels.gated_matmul(da, dg, du))
    assert rel(got, oracle.gated_matmul(a, g, u)) <= TOL_MATMUL
    np.testing.assert_array_equal(got, got2)
    np.testing.assert_array_equal(got2, kernels.download(kernels.gated_matmul(da, kernels.upload(g), kernels.upload(u))))


@pytest.mark.parametrize("m,k,n", [(1, 512, 256), (3, 1024, 1000), (8, 256, 512), (16, 640, 384), (1, 4096, 4096)])
def test_compact_weight_gemv_is_bit_identical(kernels, oracle, m, k, n):
    # src/tests_conformance.rs:2564-2640: a weight whose values are all exactly bfloat16 is kept
    # compact and gives bit-identical matmul / bias / residual results to the same values
    # stored as f32 (here: the same values in a plain, non-weight buffer).
    r = rng(24)
    a = r.standard_normal((m, k)).astype(np.float32)
    b = _bf16_exact(r.standard_normal((k, n)) / math.sqrt(k))
    bias = r.standard_normal(n).astype(np.float32)
    res = r.standard_normal((m, n)).astype(np.float32)
    da, dbias, dres = kernels.upload(a), kernels.upload(bias), kernels.upload(res)
    w = kernels.upload(b).set_weight()
    full = kernels.upload(b)
    assert not w.is_compact()
    got = kernels.download(kernels.matmul(da, w))
    assert w.is_compact() and not full.is_compact()
    np.testing.assert_array_equal(got, kernels.download(kernels.matmul(da, full)))
    assert rel(got, oracle.matmul(a, b)) <= TOL_MATMUL
    np.testing.assert_array_equal(kernels.download(kernels.matmul_bias(da, w, dbias)),
                                  kernels.download(kernels.matmul_bias(da, full, dbias)))
    np.testing.assert_array_equal(kernels.download(kernels.matmul_residual(da, w, dres)),
                                  kernels.download(kernels.matmul_residual(da, full, dres)))
    np.testing.assert_array_equal(kernels.download(w), b)  # the f32 values stay readable


@pytest.mark.parametrize("m", [1, 5, 16])
def test_compact_gated_gemv_is_bit_identical(kernels, oracle, m):
    r = rng(25)
    k, n = 768, 512
    a = r.standard_normal((m, k)).astype(np.float32)
    g = _bf16_exact(r.standard_normal((k, n)) * 0.05)
    u = _bf16_exact(r.standard_normal((k, n)) * 0.05)
    da = kernels.upload(a)
    dg, du = kernels.upload(g).set_weight(), kernels.upload(u).set_weight()
    got = kernels.download(kernels.gated_matmul(da, dg, du))
    assert dg.is_compact() and du.is_compact()
    np.testing.assert_array_equal(got, kernels.download(kernels.gated_matmul(da, kernels.upload(g), kernels.upload(u))))
    assert rel(got, oracle.gated_matmul(a, g, u)) <= TOL_MATMUL
    # one compact and one f32 weight: both stream as f32
    u2 = (r.standard_normal((k, n)) * 0.05).astype(np.float32)
    du2 = kernels.upload(u2).set_weight()
    got2 = kernels.download(kernels.gated_matmul(da, dg, du2))
    assert not du2.is_compact()
    np.testing.assert_array_equal(got2, kernels.download(kernels.gated_matmul(da, kernels.upload(g), kernels.upload(u2))))


def test_non_exact_or_small_weights_stay_f32(kernels):
    r = rng(26)
    a = r.standard_normal((2, 256)).astype(np.float32)
    da = kernels.upload(a)
    small = kernels.upload(_bf16_exact(r.standard_normal((256, 128)))).set_weight()  # 32768 values
    inexact = kernels.upload(r.standard_normal((256, 512)).astype(np.float32)).set_weight()
    kernels.matmul(da, small)
    kernels.matmul(da, inexact)
    kernels.synchronize()
    assert not small.is_compact() and not inexact.is_compact()


def test_rewriting_a_compact_weight_drops_its_compact_form(kernels, oracle):
    r = rng(27)
    a = r.standard_normal((1, 512)).astype(np.float32)
    da = kernels.upload(a)
    b = _bf16_exact(r.standard_normal((512, 256)))
    w = kernels.upload(b).set_weight()
    kernels.matmul(da, w)
    assert w.is_compact()
    b2 = r.standard_normal((512, 256)).astype(np.float32)  # not exact: stays f32 after the write
    w.write(b2)
    assert not w.is_compact()
    got = kernels.download(kernels.matmul(da, w))
    assert not w.is_compact()
    np.testing.assert_array_equal(got, kernels.download(kernels.matmul(da, kernels.upload(b2))))
    b3 = _bf16_exact(r.standard_normal((512, 256)))
    w.write(b3)
    got3 = kernels.download(kernels.matmul(da, w))
    assert w.is_compact()
    np.testing.assert_array_equal(got3, kernels.download(kernels.matmul(da, kernels.upload(b3))))


def test_greedy_select_matches_host_greedy_selection(kernels, oracle, mpc):
    # src/tests_conformance.rs:563-658: 40 seeded rounds (vocab 151936 / 1000 / 33 / 7, common
    # ties, planted NaN / inf / -inf / -0, excluded ranges, temperatures 0 / 1 / 0.7 / 1.3)
    from greedy_cases import cases
    for rnd, (logits, row, excluded, temperature) in enumerate(cases()):
        got = kernels.greedy_select(kernels.upload(logits), row, excluded, temperature)
        assert got == oracle.greedy_select(logits, row, excluded, temperature), (rnd, logits.shape, row, temperature)
    assert kernels.greedy_select(kernels.upload(np.array([[-1.0, 0.0, -0.0]], np.float32)), 0) == 1
    assert kernels.greedy_select(kernels.upload(np.array([[-1.0, -0.0, 0.0]], np.float32)), 0) == 1
    logits = kernels.upload(np.array([[1.0, np.nan, 2.0]], np.float32))
    assert kernels.greedy_select(logits, 0, [(0, 1), (2, 3)]) is None
    with pytest.raises(mpc.CudaError) as e:
        kernels.greedy_select(logits, 1)
    assert e.value.code == "ShapeUnsupported"


def test_greedy_select_many_ranges_and_wide_rows(kernels, oracle):
    r = rng(28)
    cols = 262_144
    logits = r.standard_normal((2, cols)).astype(np.float32)
    logits[1, cols - 1] = 100.0  # the last column of the last row
    d = kernels.upload(logits)
    assert kernels.greedy_select(d, 1) == cols - 1
    # more ranges than travel in the launch's parameters
    excluded = [(int(s), int(s) + 3) for s in np.argsort(-logits[0])[:40]]
    for temperature in (0.0, 0.5, 2.0):
        assert kernels.greedy_select(d, 0, excluded, temperature) == oracle.greedy_select(logits, 0, excluded, temperature)
    # every column excluded
    assert kernels.greedy_select(d, 0, [(0, cols)]) is None
    # rank-3 logits: rows are the leading dimensions flattened
    x = r.standard_normal((2, 3, 50)).astype(np.float32)
    assert kernels.greedy_select(kernels.upload(x), 4) == oracle.greedy_select(x.reshape(6, 50), 4)


def _close_scaled(actual, expected, scale):
    # src/tests_conformance.rs:3370-3379: the packed kernels sum in another order than the
    # reference CPU; |actual - expected| <= 1e-5 + 1e-5 * scale
    assert actual.shape == expected.shape
    assert np.all(np.abs(actual - expected) <= 1e-5 + 1e-5 * scale), np.max(np.abs(actual - expected))


def test_q8_packed_matmul_matches_reference_cpu(kernels, oracle):
    # src/tests_conformance.rs:3381-3438
    from q8_cases import activations, packed_q8
    k, n = 256, 96
    blocks = packed_q8(n, k, 7)  # stored as n rows of k quants: the graph sees [k, n]
    dense = oracle.q8_0_dequantize(blocks, n, k, transposed=True)
    w = kernels.upload_q8_0(blocks, n, k, transposed=True)
    assert w.is_q8() and w.is_compact() and w.shape == (k, n) and w.dtype == "q8_0"
    np.testing.assert_array_equal(kernels.download(w), dense)
    np.testing.assert_array_equal(kernels.download(kernels.dequantize_q8(w)), dense)
    bias = (np.arange(n) * 0.01).astype(np.float32)
    dbias = kernels.upload(bias)
    for m in (1, 3, 8, 16, 64, 65):
        a = activations(m, k, m)
        expected = oracle.matmul(a, dense)
        da = kernels.upload(a)
        _close_scaled(kernels.download(kernels.matmul(da, w)), expected, k)
        _close_scaled(kernels.download(kernels.matmul_bias(da, w, dbias)), expected + bias, k)
        res = activations(m, n, 99)
        _close_scaled(kernels.download(kernels.matmul_residual(da, w, kernels.upload(res))), expected + res, k)


def test_q8_packed_gated_matmul_and_embedding_match_reference_cpu(kernels, oracle):
    # src/tests_conformance.rs:4000-4040
    from q8_cases import activations, packed_q8
    k, n = 128, 64
    gate, up = packed_q8(n, k, 11), packed_q8(n, k, 12)
    dg, du = kernels.upload_q8_0(gate, n, k), kernels.upload_q8_0(up, n, k)
    g_dense = oracle.q8_0_dequantize(gate, n, k)
    u_dense = oracle.q8_0_dequantize(up, n, k)
    for m in (1, 5, 70):
        a = activations(m, k, 5)
        expected = oracle.gated_matmul(a, g_dense, u_dense)
        _close_scaled(kernels.download(kernels.gated_matmul(kernels.upload(a), dg, du)), expected, k)
    # a [vocab = 6, hidden = 64] table stored untransposed, rows read packed
    table = packed_q8(6, 64, 13)
    dt = kernels.upload_q8_0(table, 6, 64, transposed=False)
    ids = np.array([5.0, 0.0, 3.0, 5.0], np.float32)
    np.testing.assert_array_equal(kernels.download(kernels.embedding_lookup(dt, kernels.upload(ids))),
                                  oracle.embedding(oracle.q8_0_dequantize(table, 6, 64, transposed=False), ids)[0])


@pytest.mark.parametrize("m", [1, 2, 7, 16])
def test_q8_packed_matmul_at_4096(kernels, oracle, m):
    # the bench's packed lines: B [4096, 4096] stored transposed (tiled records), few rows through
    # the tensor-core form (quants widened, scaled and split in shared memory)
    r = np.random.default_rng(90 + m)
    n = k = 4096
    nb = n * k // 32
    blk = np.empty((nb, 34), np.uint8)
    blk[:, :2] = r.uniform(2.0 ** -9, 2.0 ** -5, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
    blk[:, 2:] = r.integers(-127, 128, (nb, 32), dtype=np.int8).view(np.uint8)
    w = kernels.upload_q8_0(blk.ravel(), n, k, transposed=True)
    dense = oracle.q8_0_dequantize(blk.ravel(), n, k, transposed=True)
    a = (r.standard_normal((m, k)) / math.sqrt(k)).astype(np.float32)
    got = kernels.download(kernels.matmul(kernels.upload(a), w))
    assert rel(got, oracle.matmul(a, dense)) <= TOL_MATMUL


def test_q8_packed_weights_at_real_checkpoint_sizes(kernels):
    # src/tests_conformance.rs:4128-4205: a [151936, 896] table and the same blocks as an lm head
    from q8_cases import activations, checkpoint_blocks
    vocab, hidden = 151_936, 896
    blocks, values = checkpoint_blocks(vocab, hidden)
    table = kernels.upload_q8_0(blocks, vocab, hidden, transposed=False)
    ids = [0, 1, 77_777, vocab - 1, 4242]
    rows = kernels.download(kernels.embedding_lookup(table, kernels.upload(np.array(ids, np.float32))))
    np.testing.assert_array_equal(rows, values[ids])
    lm_head = kernels.upload_q8_0(blocks, vocab, hidden, transposed=True)
    a = activations(5, hidden, 3)
    logits = kernels.download(kernels.matmul(kernels.upload(a), lm_head))
    assert logits.shape == (5, vocab)
    cols = [0, 1, 31, 32, 99_999, vocab - 1]
    expected = a.astype(np.float64) @ values[cols].T.astype(np.float64)
    assert np.all(np.abs(logits[:, cols] - expected) <= 1e-3)


def test_q8_packed_fallbacks_and_refusals(kernels, oracle, mpc):
    from q8_cases import activations, packed_q8
    # k not a multiple of 128, and untransposed storage: dequantized for the call
    for stored_rows, stored_cols, transposed, m in ((40, 96, True, 2), (96, 64, False, 3), (64, 256, False, 1)):
        blocks = packed_q8(stored_rows, stored_cols, 31)
        w = kernels.upload_q8_0(blocks, stored_rows, stored_cols, transposed=transposed)
        dense = oracle.q8_0_dequantize(blocks, stored_rows, stored_cols, transposed=transposed)
        a = activations(m, dense.shape[0], 4)
        _close_scaled(kernels.download(kernels.matmul(kernels.upload(a), w)), oracle.matmul(a, dense), dense.shape[0])
        # B transposed by the caller reads the logical matrix transposed
        at = activations(m, dense.shape[1], 6)
        _close_scaled(kernels.download(kernels.matmul(kernels.upload(at), w, transpose_b=True)),
                      oracle.matmul(at, dense.T.copy()), dense.shape[1])
    w = kernels.upload_q8_0(packed_q8(64, 128, 3), 64, 128)
    x = kernels.upload(np.ones((128, 64), np.float32))
    with pytest.raises(mpc.CudaError) as e:
        kernels.add(w, x)
    assert e.value.code == "DTypeUnsupported"
    with pytest.raises(mpc.CudaError) as e:  # rows of a transposed-storage table
        kernels.embedding_lookup(w, kernels.upload(np.array([0.0], np.float32)))
    assert e.value.code == "DTypeUnsupported"
    t = kernels.upload_q8_0(packed_q8(6, 64, 13), 6, 64, transposed=False)
    with pytest.raises(mpc.CudaError) as e:  # an id past the table
        kernels.embedding_lookup(t, kernels.upload(np.array([6.0], np.float32)))
    assert e.value.code == "ShapeUnsupported"
    with pytest.raises(mpc.CudaError) as e:  # not whole blocks
        kernels.upload_q8_0(np.zeros(33, np.uint8), 1, 32)
    assert e.value.code == "ShapeUnsupported"
    with pytest.raises(mpc.CudaError) as e:
        kernels.upload_q8_0(np.zeros(34, np.uint8), 2, 16)
    assert e.value.code == "ShapeUnsupported"
