"""GPU: the allocation-free matmul entry point (mg_matmul_gemv_fixed).

It exists for callers that cannot allocate device memory at the moment they multiply (a
runtime whose device memory is fully handed out under a fixed budget, or a latency-critical
thread that must not enter the driver's allocator).  It keeps its partial sums in a workspace
compiled into the library, so these tests check, through the C ABI, that calls in a row
match the CPU oracle's matmul (and an f64 product) within the matmul tolerance, and that a shape whose
partials would not fit the fixed workspace is refused with a clear error.  The file name
sorts last so that a run stopping at the first failure has run every other test before it.
"""
import ctypes
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL_MATMUL = 1e-4  # relative L2, the matmul bar of the other GPU tests


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def fixed_gemv(mpc, kernels, a_buf, b_buf, out_buf, m, k, n):
    lib = mpc.lib()
    status = lib.mg_matmul_gemv_fixed(kernels.ordinal, ctypes.c_void_p(kernels.stream),
                                      ctypes.c_void_p(a_buf.data_ptr()), ctypes.c_void_p(b_buf.data_ptr()),
                                      ctypes.c_void_p(out_buf.data_ptr()), m, k, n)
    return status


@pytest.mark.parametrize("shapes", [[(16, 4096, 4096), (3, 1000, 256)], [(1, 512, 1376), (16, 512, 1376)],
                                    [(5, 777, 260), (7, 4099, 1028)]])
def test_fixed_workspace_gemv_matches_the_oracle(mpc, kernels, oracle, shapes):
    # Odd row counts and k that is not a multiple of the kernel's k step (ragged slices) too.
    r = np.random.default_rng(42)
    for m, k, n in shapes:  # two calls in a row share the fixed workspace
        a = (r.standard_normal((m, k)) / math.sqrt(k)).astype(np.float32)
        b = r.standard_normal((k, n)).astype(np.float32)
        da, db = kernels.upload(a), kernels.upload(b)
        out = kernels.empty((m, n))
        assert fixed_gemv(mpc, kernels, da, db, out, m, k, n) == 0, mpc.lib().mg_last_error()
        got = kernels.download(out)
        assert rel(got, oracle.matmul(a, b)) <= TOL_MATMUL
        assert rel(got, a.astype(np.float64) @ b.astype(np.float64)) <= TOL_MATMUL


def test_fixed_workspace_gemv_refuses_shapes_beyond_its_workspace(mpc, kernels):
    m, k, n = 16, 32, 262144  # partials of 16 x 262144 floats exceed 8 MiB
    da = kernels.upload(np.ones((m, k), np.float32))
    db = kernels.upload(np.ones((k, n), np.float32))
    out = kernels.empty((m, n))
    status = fixed_gemv(mpc, kernels, da, db, out, m, k, n)
    assert status == 1  # MG_SHAPE_UNSUPPORTED
    assert b"fixed workspace holds" in mpc.lib().mg_last_error()
    assert fixed_gemv(mpc, kernels, da, db, out, 17, k, 256) == 1  # more than 16 rows
