"""Generates ``tests/golden/ref_ops.npz``: seeded inputs and the outputs of the reference's own
per-op CUDA kernels on them (run on a GPU box from the repo root, after ``make -C oracle ref``
has compiled the reference's ``src/kernels.cu`` into ``oracle/_ref/``):

    python tests/golden/make_ref_golden.py [out.npz]

The kernels run through ``oracle/ref_kernels.py`` with the reference's launch shapes and
arguments.  ``tests/test_oracle.py`` then checks the CPU oracle against these outputs on the
same inputs, which pins the oracle's f32 restatement (add, mul, silu, silu-mul, gelu, sigmoid,
embedding, rmsnorm, rope, softmax, matmul, attention, half add/mul) to the reference itself.
Sizes are small so that the oracle reproduces every case in seconds on the CPU.
"""
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)


def cases():
    """(name, op, inputs, kwargs) for every fixture; inputs are float32 (or uint16) arrays."""
    r = np.random.default_rng(20261202)

    def n(*shape, s=1.0):
        return (r.standard_normal(shape) * s).astype(np.float32)

    out = []
    # elementwise (src/kernels.cu:30-117, 1079-1084): values with infinities, NaN, subnormals
    a, b = n(37, 129), n(37, 129)
    a[0, :6] = [np.inf, -np.inf, np.nan, 1e-40, -0.0, 3e38]
    b[0, :6] = [1.0, np.inf, 2.0, 1e-40, 0.0, 3e38]
    out += [("add", "add", [a, b], {}), ("mul", "mul", [a, b], {})]
    x = n(32, 257, s=3.0)
    x[0, :5] = [90.0, -90.0, 0.0, -0.0, 1e-30]
    out += [("silu", "silu", [x], {}), ("gelu", "gelu_tanh", [x], {}), ("sigmoid", "sigmoid", [x], {}),
            ("silu_mul", "silu_mul", [x, n(32, 257)], {})]
    # embedding (src/kernels.cu:127-176)
    table = n(100, 48)
    ids = r.integers(0, 100, 29).astype(np.float32)
    out.append(("embedding", "embedding", [table, ids], {}))
    bad = ids.copy()
    bad[[3, 7, 11]] = [100.0, -1.0, 2.5]
    out.append(("embedding_invalid", "embedding", [table, bad], {}))
    # rmsnorm (src/kernels.cu:1104-1138)
    out.append(("rmsnorm_gain", "rmsnorm", [n(33, 300), (1 + 0.1 * n(300))], {"epsilon": 1e-5}))
    out.append(("rmsnorm_plain", "rmsnorm", [n(16, 1024, s=4.0)], {"epsilon": 1e-6}))
    out.append(("rmsnorm_heads", "rmsnorm", [n(8, 256), (1 + 0.1 * n(64))], {"epsilon": 1e-5, "heads": [4, 64]}))
    out.append(("rmsnorm_wide", "rmsnorm", [n(3, 5000), (1 + 0.1 * n(5000))], {"epsilon": 1e-5}))
    # rope (src/kernels.cu:1147-1229)
    out.append(("rope_interleaved", "rope", [n(40, 512)], {"base": 10000.0, "dimension": 64, "head_count": 8}))
    out.append(("rope_half_split_offset", "rope", [n(24, 512)],
                 {"base": 500000.0, "dimension": 128, "head_count": 4, "position_offset": 1000, "half_split": True}))
    out.append(("rope_banded", "rope", [n(16, 256)],
                 {"base": 500000.0, "dimension": 128, "head_count": 2, "position_offset": 5000,
                  "banded": [8.0, 1.0, 4.0, 8192.0]}))
    out.append(("rope_yarn", "rope", [n(16, 256)],
                 {"base": 10000.0, "dimension": 64, "head_count": 4, "position_offset": 300,
                  "yarn": [4.0, 10.0, 25.0, 1.2]}))
    out.append(("rope_partial", "rope", [n(12, 384)],
                 {"base": 10000.0, "dimension": 64, "head_count": 4, "rotated_pairs": 16, "scale": 0.5}))
    # softmax (src/kernels.cu:1232-1260)
    s = n(50, 333, s=2.0)
    s[1, :100] = -np.inf
    out.append(("softmax", "softmax", [s], {}))
    s2 = n(4, 64)
    s2[2, :] = -np.inf
    out.append(("softmax_nonfinite_row", "softmax", [s2], {}))
    # matmul (src/kernels.cu:1265-1294): k ascending, transposes by strides
    out.append(("matmul_small", "matmul", [n(7, 65), n(65, 33)], {}))
    out.append(("matmul_rows16", "matmul", [n(16, 256), n(256, 130)], {}))
    out.append(("matmul_row1_k1000", "matmul", [n(1, 1000), n(1000, 64)], {}))
    out.append(("matmul_ta", "matmul", [n(40, 9), n(40, 17)], {"transpose_a": True}))
    out.append(("matmul_tb", "matmul", [n(9, 40), n(17, 40)], {"transpose_b": True}))
    out.append(("matmul_ta_tb", "matmul", [n(40, 9), n(17, 40)], {"transpose_a": True, "transpose_b": True}))
    out.append(("matmul_m128_k512", "matmul", [n(128, 512), n(512, 64, s=0.05)], {}))
    # attention (src/kernels.cu:1873-1959)
    H, D = 8, 64
    out.append(("attention_causal", "attention", [n(40, H * D), n(40, H * D), n(40, H * D)],
                 {"head_count": H, "head_dimension": D, "causal": True}))
    out.append(("attention_gqa_offset", "attention", [n(20, 8 * 32), n(50, 2 * 32), n(50, 2 * 32)],
                 {"head_count": 8, "head_dimension": 32, "kv_head_count": 2, "causal": True}))
    out.append(("attention_window", "attention", [n(30, 4 * 32), n(30, 4 * 32), n(30, 4 * 32)],
                 {"head_count": 4, "head_dimension": 32, "causal": True, "window_size": 5}))
    out.append(("attention_bidirectional_scale", "attention", [n(17, 2 * 64), n(23, 2 * 64), n(23, 2 * 64)],
                 {"head_count": 2, "head_dimension": 64, "causal": False, "scale": 0.3}))
    out.append(("attention_key_count", "attention", [n(1, 4 * 32), n(64, 4 * 32), n(64, 4 * 32)],
                 {"head_count": 4, "head_dimension": 32, "causal": True, "key_count": 37}))
    out.append(("attention_value_dim", "attention", [n(12, 2 * 32), n(12, 2 * 32), n(12, 2 * 48)],
                 {"head_count": 2, "head_dimension": 32, "causal": True, "value_dimension": 48}))
    out.append(("attention_d128_s160", "attention", [n(160, 2 * 128), n(160, 2 * 128), n(160, 2 * 128)],
                 {"head_count": 2, "head_dimension": 128, "causal": True}))
    # half add / mul (src/kernels.cu:2806-2939) on random 16-bit patterns
    for dt in ("f16", "bf16"):
        ha = r.integers(0, 1 << 16, 4096, dtype=np.uint32).astype(np.uint16)
        hb = r.integers(0, 1 << 16, 4096, dtype=np.uint32).astype(np.uint16)
        for op in ("add", "mul"):
            out.append((f"half_{op}_{dt}", "half_binary", [ha, hb], {"dtype": dt, "op": op}))
    return out


def run_reference(op, inputs, kw):
    """The reference kernel's output (and flag, where the kernel has one) as numpy."""
    from oracle import ref_kernels as rk
    fn = getattr(rk, op)
    res = fn(*inputs, **kw)
    if isinstance(res, tuple):
        return res[0].cpu().numpy(), bool(res[1])
    t = res.cpu().numpy()
    if op == "half_binary":
        t = t.view(np.uint16)
    return t, None


def main():
    path = sys.argv[1] if len(sys.argv) > 1 else os.path.join(ROOT, "tests", "golden", "ref_ops.npz")
    arrays, manifest = {}, []
    for name, op, inputs, kw in cases():
        outv, flag = run_reference(op, inputs, kw)
        for i, x in enumerate(inputs):
            arrays[f"{name}/in{i}"] = x
        arrays[f"{name}/out"] = outv
        manifest.append({"name": name, "op": op, "inputs": len(inputs), "kwargs": kw, "flag": flag})
    arrays["manifest"] = np.frombuffer(json.dumps({
        "source": "outputs of the reference's src/kernels.cu kernels (compiled by oracle/Makefile `ref`), "
                  "launched as src/kernels.rs launches them, by tests/golden/make_ref_golden.py",
        "cases": manifest}).encode(), dtype=np.uint8)
    np.savez_compressed(path, **arrays)
    print(f"wrote {len(manifest)} cases to {path}")


if __name__ == "__main__":
    main()
