"""One rank of the multi-GPU tensor-parallel parity check (launched by test_tp_ranks_gpu.py
with torch.distributed.run, one process per GPU).

Every rank builds the same full weights from one seed, keeps its shares (gate/up by columns,
down by rows, the reference's ``WeightShard`` split, src/multi/tensor_parallel.rs:300-307),
and runs
  1. the tensor-parallel SwiGLU MLP entry point (one NCCL all-reduce, chunked), and
  2. the executor with a tensor-parallel plan (``apply_tensor_parallel``: its row-split
     matmul all-reduces the partial outputs, src/multi.rs:543-562), run directly and
     captured as one step whose graph holds the all-reduce, replayed with new inputs,
then compares its result with the CPU oracle of the unsplit computation (rel-L2 <= 1e-4).
A rank that fails exits non-zero; the process group has a short timeout so that the others
end with an error instead of waiting.
"""
import datetime
import importlib
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def main():
    import torch
    import torch.distributed as dist

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", local))
    mpc = importlib.import_module("magnetar-provider-cuda_b200")
    tp = importlib.import_module("magnetar-provider-cuda_b200.tensor_parallel")
    from oracle import oracle as orc

    results = {}
    kernels = mpc.CudaKernels(local)
    group = tp.TpGroup.from_torch_distributed(kernels)
    try:
        r = np.random.default_rng(2024)
        for tokens, hidden, ffn in ((256, 512, 1376), (100, 256, 700)):
            x = r.standard_normal((tokens, hidden)).astype(np.float32)
            wg = (r.standard_normal((hidden, ffn)) * 0.02).astype(np.float32)
            wu = (r.standard_normal((hidden, ffn)) * 0.02).astype(np.float32)
            wd = (r.standard_normal((ffn, hidden)) * 0.02).astype(np.float32)
            exp = orc.matmul(orc.gated_matmul(x, wg, wu), wd)
            for chunks in (1, 4):
                y = group.mlp(kernels.upload(x), kernels.upload(tp.split_columns(wg, world, rank)),
                              kernels.upload(tp.split_columns(wu, world, rank)),
                              kernels.upload(tp.split_rows(wd, world, rank)), chunks=chunks)
                results[f"mlp t{tokens} h{hidden} f{ffn} chunks{chunks}"] = rel(kernels.download(y), exp)

        # the executor's plan: "up" column-split, "down" row-split (all-reduced)
        ex = mpc.CudaExecutor(kernels)
        try:
            ex.attach_comm(group)
            ex.apply_tensor_parallel({"up": "columns", "down": "rows"})
            x = r.standard_normal((16, 128)).astype(np.float32)
            up = r.standard_normal((128, 320)).astype(np.float32)
            down = r.standard_normal((320, 128)).astype(np.float32)
            ex.write_tensor("x", x)
            ex.write_weight_tensor("up", up)
            ex.write_weight_tensor("down", down)
            ex.run(mpc.KernelInvocation("matmul", ["x", "up"], "h"))
            ex.run(mpc.KernelInvocation("matmul", ["h", "down"], "y"))
            results["executor plan up=columns down=rows"] = rel(ex.read_tensor("y"),
                                                                orc.matmul(orc.matmul(x, up), down))
            # the same two matmuls captured as one step under the plan, the all-reduce of the
            # row-split projection inside the graph (src/multi/tensor_parallel.rs:542-690), then
            # replayed with new inputs written into the captured buffer
            ex.begin_step_capture()
            ex.run(mpc.KernelInvocation("matmul", ["x", "up"], "h"))
            ex.run(mpc.KernelInvocation("matmul", ["h", "down"], "y"))
            step = ex.end_step_capture_id()
            results["captured plan, first run"] = rel(ex.read_tensor("y"), orc.matmul(orc.matmul(x, up), down))
            for t in range(3):
                xt = np.random.default_rng(77 + t).standard_normal((16, 128)).astype(np.float32)
                yt = np.empty((16, 128), np.float32)
                ex.replay_capture(step, inputs={"x": xt}, outputs={"y": yt})
                results[f"captured plan, replay {t}"] = rel(yt, orc.matmul(orc.matmul(xt, up), down))
            ex.release_step_capture(step)
            ex.attach_comm(None)
        finally:
            ex.close()
    finally:
        group.close()
        kernels.close()
    ok = all(v <= 1e-4 for v in results.values())
    print(json.dumps({"rank": rank, "world": world, "ok": ok, "rel_l2": results}), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
