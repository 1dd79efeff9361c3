"""CPU, world size 2 over gloo: the tensor-parallel MLP's host logic -- each rank keeps its
column shares of gate/up and its row share of down, computes its partial output, and the
sum across ranks equals the unsplit MLP.  The per-rank compute here is the oracle (this
test checks the sharding and reduction plan, the GPU tests check the kernels)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, tokens, hidden, ffn, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import importlib
    from datetime import timedelta
    from oracle import oracle as orc
    tp = importlib.import_module("magnetar-provider-cuda_b200.tensor_parallel")
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    rng = np.random.default_rng(0)
    x = rng.standard_normal((tokens, hidden)).astype(np.float32)
    wg = (rng.standard_normal((hidden, ffn)) * 0.02).astype(np.float32)
    wu = (rng.standard_normal((hidden, ffn)) * 0.02).astype(np.float32)
    wd = (rng.standard_normal((ffn, hidden)) * 0.02).astype(np.float32)
    g_s = tp.split_columns(wg, world, rank)
    u_s = tp.split_columns(wu, world, rank)
    d_s = tp.split_rows(wd, world, rank)
    h = orc.gated_matmul(x, g_s, u_s)
    partial = torch.from_numpy(orc.matmul(h, d_s))
    dist.all_reduce(partial)
    if rank == 0:
        full = orc.matmul(orc.gated_matmul(x, wg, wu), wd)
        np.save(result_path, np.stack([partial.numpy(), full]))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("ffn", [256, 100])
def test_tp_mlp_partials_sum_to_the_full_mlp(tmp_path, ffn):
    world, tokens, hidden = 2, 16, 64
    path = str(tmp_path / "r.npy")
    mp.start_processes(_worker, args=(world, _free_port(), tokens, hidden, ffn, path), nprocs=world,
                       join=True, start_method="spawn")
    got, full = np.load(path)
    rel = np.linalg.norm(got - full) / np.linalg.norm(full)
    assert rel < 1e-5, rel
