"""Generates the committed golden fixtures under tests/golden/ (run from the repo root:
``python tests/golden/make_golden.py``).

The reference's own pinned vectors for the half-precision path are the literal inputs of
its bit-exact tests (src/tests_conformance.rs:2349-2423: a = [1, 2.5, 3, -4.25, 0.1, 100],
b = [6, 0.2, 4, 3, 0.2, -99.5]) with expectations from its half_precision model
(src/half_precision.rs).  The expectations here are computed with independent IEEE
implementations -- numpy's float16 and torch's bfloat16 conversions, both round-to-nearest-
even -- so that the oracle's own restatement is checked against something it does not share
code with.  NaN payload rules are reference-specific and are pinned separately by the
exhaustive round-trip property test.  The TP share vectors are the reference's unit-test
expectations (src/multi/tensor_parallel.rs:755-848).
"""
import json
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

A = [1.0, 2.5, 3.0, -4.25, 0.1, 100.0]
B = [6.0, 0.2, 4.0, 3.0, 0.2, -99.5]
# Extra edge values: subnormal, overflow, signed zeros, infinities, rounding ties.
A_EDGE = [6.0e-8, 65504.0, -0.0, float("inf"), 1.0009765625, 3.0e38, 1e-40, -2.0, 0.333333343]
B_EDGE = [6.0e-8, 65504.0, 0.0, 1.0, 2.0 ** -11, 3.0e38, 1e-40, 0.5, 3.0]


def f16_bits(x):
    return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def f16_vals(bits):
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


def bf16_bits(x):
    t = torch.tensor(np.asarray(x, dtype=np.float32)).to(torch.bfloat16)
    return t.view(torch.int16).numpy().view(np.uint16)


def bf16_vals(bits):
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def case(a, b, dtype, op):
    enc, dec = (f16_bits, f16_vals) if dtype == "f16" else (bf16_bits, bf16_vals)
    ab, bb = enc(a), enc(b)
    x, y = dec(ab), dec(bb)
    r = (x + y) if op == "add" else (x * y)
    rb = enc(r.astype(np.float32))
    return {"dtype": dtype, "op": op, "a_f32": [float(v) for v in a], "b_f32": [float(v) for v in b],
            "a_bits": ab.tolist(), "b_bits": bb.tolist(), "out_bits": rb.tolist()}


def main():
    cases = []
    for dtype in ("f16", "bf16"):
        for op in ("add", "mul"):
            cases.append(case(A, B, dtype, op))
            cases.append(case(A_EDGE, B_EDGE, dtype, op))
    with open(os.path.join(HERE, "half_ops.json"), "w") as f:
        json.dump({"source": "src/tests_conformance.rs:2349-2423 inputs; numpy float16 / torch bfloat16 RNE",
                   "cases": cases}, f, indent=1)
    tp = {
        "source": "src/multi/tensor_parallel.rs:755-848",
        "share_granule": [[64, 2, 32], [48, 2, 1]],
        "local_extent": [[64, 2, 1, 32], [7, 2, 1, 4]],
        "split_2x6": {"columns": [[0, 1, 2, 6, 7, 8], [3, 4, 5, 9, 10, 11]], "rows0": [0, 1, 2, 3, 4, 5],
                      "bias_columns1": [3, 4, 5]},
        "expert_range_5_of_2": [[0, 2], [2, 5]],
    }
    with open(os.path.join(HERE, "tp_shares.json"), "w") as f:
        json.dump(tp, f, indent=1)


if __name__ == "__main__":
    main()
