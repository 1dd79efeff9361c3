"""GPU: the tensor-parallel MLP entry point on one rank (a group of one) against the oracle,
and the executor's plan on a single rank.  Multi-rank runs go through bench.py --gpus N."""
import importlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("chunks", [1, 4])
def test_tp_mlp_single_rank(kernels, oracle, chunks):
    tp = importlib.import_module("magnetar-provider-cuda_b200.tensor_parallel")
    r = np.random.default_rng(0)
    tokens, hidden, ffn = 256, 512, 1024
    x = r.standard_normal((tokens, hidden)).astype(np.float32)
    wg = (r.standard_normal((hidden, ffn)) * 0.02).astype(np.float32)
    wu = (r.standard_normal((hidden, ffn)) * 0.02).astype(np.float32)
    wd = (r.standard_normal((ffn, hidden)) * 0.02).astype(np.float32)
    g = tp.TpGroup(kernels, 0, 1, tp.TpGroup.unique_id())
    try:
        y = g.mlp(kernels.upload(x), kernels.upload(wg), kernels.upload(wu), kernels.upload(wd), chunks=chunks)
        exp = oracle.matmul(oracle.gated_matmul(x, wg, wu), wd)
        assert rel(kernels.download(y), exp) <= 1e-4
    finally:
        g.close()


def test_tp_mlp_timing_split(kernels, oracle, mpc):
    # the measurement hook: start -> last down chunk, then the exposed all-reduce; results unchanged
    tp = importlib.import_module("magnetar-provider-cuda_b200.tensor_parallel")
    r = np.random.default_rng(5)
    x = r.standard_normal((512, 256)).astype(np.float32)
    wg = (r.standard_normal((256, 768)) * 0.05).astype(np.float32)
    wu = (r.standard_normal((256, 768)) * 0.05).astype(np.float32)
    wd = (r.standard_normal((768, 256)) * 0.05).astype(np.float32)
    g = tp.TpGroup(kernels, 0, 1, tp.TpGroup.unique_id())
    try:
        args = [kernels.upload(v) for v in (x, wg, wu, wd)]
        with pytest.raises(mpc.CudaError):
            g.mlp_timing()  # timing is off
        g.set_mlp_timing(True)
        with pytest.raises(mpc.CudaError):
            g.mlp_timing()  # on, but nothing timed yet
        y = g.mlp(*args, chunks=4)
        compute_ms, exposed_ms = g.mlp_timing()
        assert compute_ms > 0.0 and 0.0 <= exposed_ms < compute_ms
        assert rel(kernels.download(y), oracle.matmul(oracle.gated_matmul(x, wg, wu), wd)) <= 1e-4
        g.set_mlp_timing(False)
        g.mlp(*args, chunks=4)
        with pytest.raises(mpc.CudaError):
            g.mlp_timing()
    finally:
        g.close()


def test_executor_plan_on_one_rank(executor, oracle):
    tp = importlib.import_module("magnetar-provider-cuda_b200.tensor_parallel")
    mpc = importlib.import_module("magnetar-provider-cuda_b200")
    g = tp.TpGroup(executor.kernels, 0, 1, tp.TpGroup.unique_id())
    try:
        executor.attach_comm(g)
        executor.apply_tensor_parallel({"up": "columns", "down": "rows"})
        r = np.random.default_rng(1)
        x = r.standard_normal((8, 64)).astype(np.float32)
        up = r.standard_normal((64, 96)).astype(np.float32)
        down = r.standard_normal((96, 64)).astype(np.float32)
        executor.write_tensor("x", x)
        executor.write_weight_tensor("up", up)
        executor.write_weight_tensor("down", down)
        executor.run(mpc.KernelInvocation("matmul", ["x", "up"], "h"))
        executor.run(mpc.KernelInvocation("matmul", ["h", "down"], "y"))
        assert rel(executor.read_tensor("y"), oracle.matmul(oracle.matmul(x, up), down)) <= 1e-4
    finally:
        executor.attach_comm(None)
        g.close()
