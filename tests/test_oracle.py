"""CPU: the oracle pinned against the reference's golden vectors and closed-form answers."""
import json
import math
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_f16_round_trips_every_bit_pattern(oracle):
    # src/half_precision.rs:136-148
    for bits in range(65536):
        v = oracle.f16_to_f32(bits)
        back = oracle.f32_to_f16(v)
        if math.isnan(v):
            assert math.isnan(oracle.f16_to_f32(back))
        else:
            assert back == bits, hex(bits)


def test_bf16_round_trips_every_bit_pattern(oracle):
    # src/half_precision.rs:150-162
    for bits in range(65536):
        v = oracle.bf16_to_f32(bits)
        back = oracle.f32_to_bf16(v)
        if math.isnan(v):
            assert math.isnan(oracle.bf16_to_f32(back))
        else:
            assert back == bits, hex(bits)


def test_half_nan_payload_rules(oracle):
    # src/half_precision.rs:53-59, 109-114: the payload's top bits survive, zero becomes 1/0x40
    f32 = np.array([0x7FC00000, 0xFF800001, 0x7F802000, 0x7FFFFFFF, 0x7F800001], dtype=np.uint32).view(np.float32)
    assert oracle.encode_half(f32, "f16").tolist() == [0x7E00, 0xFC01, 0x7C01, 0x7FFF, 0x7C01]
    assert oracle.encode_half(f32, "bf16").tolist() == [0x7FC0, 0xFFC0, 0x7FC0, 0x7FFF, 0x7FC0]
    back = oracle.decode_half(np.array([0x7C01, 0xFE00, 0x7F81], np.uint16), "f16").view(np.uint32)
    assert back.tolist() == [0x7F802000, 0xFFC00000, 0x7FF02000]


def test_half_ops_match_golden_vectors(oracle):
    cases = json.load(open(os.path.join(GOLDEN, "half_ops.json")))["cases"]
    for c in cases:
        a = np.array(c["a_bits"], dtype=np.uint16)
        b = np.array(c["b_bits"], dtype=np.uint16)
        assert oracle.encode_half(np.array(c["a_f32"], np.float32), c["dtype"]).tolist() == c["a_bits"]
        out = oracle.half_binary(a, b, c["dtype"], c["op"])
        assert out.tolist() == c["out_bits"], c
        # the executor's f32-resident form gives the decoded same bits
        f = oracle.half_binary_f32(np.array(c["a_f32"], np.float32), np.array(c["b_f32"], np.float32),
                                   c["dtype"], c["op"])
        np.testing.assert_array_equal(f.view(np.uint32),
                                      oracle.decode_half(np.array(c["out_bits"], np.uint16), c["dtype"]).view(np.uint32))


def test_matmul_keeps_f32_activation_precision(oracle):
    # src/tests_conformance.rs:820-846: a = 1 + 2^-12 everywhere, |b| bf16-exact
    m, k, n = 7, 90, 13
    a = np.full((m, k), 1.0 + 2.0 ** -12, np.float32)
    rng = np.random.default_rng(21)
    w = np.abs(rng.standard_normal((k, n)).astype(np.float32))
    w = (w.view(np.uint32) & 0xFFFF0000).view(np.float32)
    out = oracle.matmul(a, w)
    expected = (1.0 + 2.0 ** -12) * w.astype(np.float64).sum(axis=0)
    assert np.all(np.abs(out - expected) <= 5e-5 * expected)


def test_matmul_near_f32_max_stays_finite(oracle):
    # src/tests_conformance.rs:852-880
    m, k, n = 4, 256, 8
    a = np.full((m, k), np.finfo(np.float32).max, np.float32)
    b = np.full((k, n), 2.0 ** -120, np.float32)
    out = oracle.matmul(a, b)
    expected = float(np.finfo(np.float32).max) * 2.0 ** -120 * k
    assert np.all(np.isfinite(out)) and np.all(np.abs(out / expected - 1) < 1e-4)


def test_attention_large_values_stay_finite(oracle):
    # src/tests_conformance.rs:884-914: q = k = 0, v = 1e38 -> every output 1e38
    rows = 70
    q = np.zeros((rows, 64), np.float32)
    v = np.full((rows, 64), 1e38, np.float32)
    out = oracle.attention(q, q, v, 1, 64, causal=True)
    assert np.all(np.isfinite(out)) and np.all(np.abs(out / 1e38 - 1) < 1e-4)


def test_causal_attention_small_case(oracle):
    # src/tests_conformance.rs:946-968 inputs; the expectation written out from the definition
    q = np.array([[1, 0], [0, 1], [1, 1]], np.float32)
    k = np.array([[1, 0], [0, 1], [0.5, 0.5]], np.float32)
    v = np.array([[1, 2], [3, 4], [5, 6]], np.float32)
    out = oracle.attention(q, k, v, 1, 2, causal=True)
    s = 1 / math.sqrt(2)
    exp = np.zeros((3, 2))
    for i in range(3):
        sc = np.array([q[i] @ k[j] * s for j in range(i + 1)])
        w = np.exp(sc - sc.max())
        w /= w.sum()
        exp[i] = w @ v[: i + 1]
    np.testing.assert_allclose(out, exp, rtol=1e-6, atol=1e-6)


def test_embedding_flags_invalid_ids(oracle):
    table = np.arange(12, dtype=np.float32).reshape(4, 3)
    rows, bad = oracle.embedding(table, np.array([1, 3, 0], np.float32))
    assert not bad and rows.tolist() == [[3, 4, 5], [9, 10, 11], [0, 1, 2]]
    for ids in ([4.0], [-1.0], [1.5], [float("nan")]):
        _, bad = oracle.embedding(table, np.array(ids, np.float32))
        assert bad, ids


def test_softmax_flags_non_finite_rows(oracle):
    x = np.array([[1, 2, 3], [-np.inf, -np.inf, -np.inf]], np.float32)
    _, flag = oracle.softmax(x)
    assert flag
    out, flag = oracle.softmax(x[:1])
    assert not flag
    np.testing.assert_allclose(out.sum(), 1.0, rtol=1e-6)


def test_rope_pairings_rotate_by_position(oracle):
    # 3 rows, 2 heads of width 6, dimension 4 (partial): src/tests_conformance.rs:2449-2470 shape
    x = (np.arange(36, dtype=np.float32) * 0.07 - 1.2).reshape(3, 12)
    for half_split in (False, True):
        out = oracle.rope(x, dimension=4, head_count=2, half_split=half_split)
        np.testing.assert_array_equal(out[0], x[0])  # position 0: identity
        np.testing.assert_array_equal(out[:, 4:6], x[:, 4:6])  # untouched tail of head 0
        assert not np.array_equal(out[1], x[1])


def test_rmsnorm_matches_definition(oracle):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((5, 300)).astype(np.float32)
    w = rng.standard_normal(300).astype(np.float32)
    out = oracle.rmsnorm(x, w, 1e-5)
    ref = x / np.sqrt((x.astype(np.float64) ** 2).mean(axis=1, keepdims=True) + 1e-5) * w
    np.testing.assert_allclose(out, ref, rtol=2e-6, atol=1e-6)


def test_oracle_layered_forms_against_numpy(oracle):
    # gelu (tanh), sigmoid, softcap, row-scale, concat across heads and batched-matmul: the C
    # restatements against independent float64 numpy computations of the same definitions.
    r = np.random.default_rng(31)
    x = (r.standard_normal((7, 40)) * 4).astype(np.float32)
    x64 = x.astype(np.float64)
    gelu = 0.5 * x64 * (1 + np.tanh(0.7978846 * (x64 + 0.044715 * x64 ** 3)))
    np.testing.assert_allclose(oracle.gelu_tanh(x), gelu, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(oracle.sigmoid(x), 1 / (1 + np.exp(-x64)), rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(oracle.softcap(x, 1.5), 1.5 * np.tanh(x64 / 1.5), rtol=1e-6, atol=1e-6)
    s = r.standard_normal(7).astype(np.float32)
    np.testing.assert_array_equal(oracle.row_scale(x, s), x * s[:, None])
    a = r.standard_normal((5, 4 * 6)).astype(np.float32)
    b = r.standard_normal((5, 4 * 2)).astype(np.float32)
    exp = np.concatenate([a.reshape(5, 4, 6), b.reshape(5, 4, 2)], axis=2).reshape(5, 32)
    np.testing.assert_array_equal(oracle.concat_heads(a, b, 4), exp)
    b1 = r.standard_normal((5, 3)).astype(np.float32)
    exp1 = np.concatenate([a.reshape(5, 4, 6), np.repeat(b1[:, None, :], 4, axis=1)], axis=2).reshape(5, 36)
    np.testing.assert_array_equal(oracle.concat_heads(a, b1, 4, 1), exp1)
    ga = r.standard_normal((3, 2 * 8)).astype(np.float32)
    gb = r.standard_normal((2 * 8, 5)).astype(np.float32)
    exp = np.concatenate([ga[:, g * 8:(g + 1) * 8].astype(np.float64) @ gb[g * 8:(g + 1) * 8] for g in range(2)], axis=1)
    np.testing.assert_allclose(oracle.batched_matmul(ga, gb, 2), exp, rtol=1e-5, atol=1e-5)
    gbt = r.standard_normal((2 * 5, 8)).astype(np.float32)
    exp = np.concatenate([ga[:, g * 8:(g + 1) * 8].astype(np.float64) @ gbt[g * 5:(g + 1) * 5].T for g in range(2)],
                         axis=1)
    np.testing.assert_allclose(oracle.batched_matmul(ga, gbt, 2, transpose_b=True), exp, rtol=1e-5, atol=1e-5)


def test_greedy_select_oracle_matches_the_host_rule(oracle):
    from greedy_cases import cases, host_greedy
    for logits, row, excluded, temperature in cases(rounds=24, widths=(2000, 1000, 33, 7)):
        assert oracle.greedy_select(logits, row, excluded, temperature) == host_greedy(logits[row], excluded, temperature)
    # -0 and +0 compare equal: the lower column wins (src/tests_conformance.rs:630-645)
    assert oracle.greedy_select(np.array([[-1.0, 0.0, -0.0]], np.float32), 0) == 1
    assert oracle.greedy_select(np.array([[-1.0, -0.0, 0.0]], np.float32), 0) == 1
    # nothing eligible
    assert oracle.greedy_select(np.array([[1.0, np.nan, 2.0]], np.float32), 0, [(0, 1), (2, 3)]) is None


def test_q8_0_dequantize_known_answers(oracle):
    from q8_cases import checkpoint_blocks, packed_q8
    blocks, values = checkpoint_blocks(6, 64)
    np.testing.assert_array_equal(oracle.q8_0_dequantize(blocks, 6, 64, transposed=False), values)
    np.testing.assert_array_equal(oracle.q8_0_dequantize(blocks, 6, 64, transposed=True), values.T)
    # against numpy's own f16 widening of the scales
    raw = packed_q8(8, 96, 7).reshape(-1, 34)
    d = raw[:, :2].copy().view(np.float16).astype(np.float32).ravel()
    q = raw[:, 2:].view(np.int8).astype(np.float32)
    np.testing.assert_array_equal(oracle.q8_0_dequantize(raw, 8, 96, transposed=False), (q * d[:, None]).reshape(8, 96))
    assert q.min() >= -127 and q.max() <= 127 and (q.min(), q.max()) != (0, 0)


# ---- the oracle against the reference's own kernels -------------------------------------------
# tests/golden/ref_ops.npz holds seeded inputs and the outputs of the reference's src/kernels.cu
# kernels on them, run on a B200 by tests/golden/make_ref_golden.py (oracle/ref_kernels.py
# launches each kernel as src/kernels.rs does).  Exact operations must agree bit for bit; the
# others differ only in rounding (the GPU's expf / sinf / cosf / powf, and where each compiler
# contracts a multiply-add), far inside the bars the provider is held to.
REF_BITEXACT = {"add", "mul", "embedding", "half_binary"}
REF_TOL = {"matmul": 1e-6, "attention": 1e-6}  # rel-L2; every other op 1e-6 too, stated per case below
REF_FIXTURE = os.path.join(GOLDEN, "ref_ops.npz")


def _ref_cases():
    if not os.path.exists(REF_FIXTURE):
        return []
    z = np.load(REF_FIXTURE)
    manifest = json.loads(bytes(z["manifest"]).decode())
    return [(c, z) for c in manifest["cases"]]


def _oracle_run(oracle, op, inputs, kw):
    fn = getattr(oracle, op)
    if op == "half_binary":
        return fn(inputs[0], inputs[1], kw["dtype"], kw["op"]), None
    kw = dict(kw)
    if op == "rmsnorm" and "heads" in kw:
        kw["heads"] = tuple(kw["heads"])
    for key in ("banded", "yarn"):
        if key in kw:
            kw[key] = tuple(kw[key])
    res = fn(*inputs, **kw)
    return (res[0], res[1]) if isinstance(res, tuple) else (res, None)


def test_reference_fixture_covers_every_f32_op():
    ops = {c["op"] for c, _ in _ref_cases()}
    assert ops >= {"add", "mul", "silu", "silu_mul", "gelu_tanh", "sigmoid", "embedding", "rmsnorm", "rope",
                   "softmax", "matmul", "attention", "half_binary"}, ops


@pytest.mark.parametrize("case", [c["name"] for c, _ in _ref_cases()])
def test_oracle_matches_the_reference_kernels(oracle, case):
    c, z = next((c, z) for c, z in _ref_cases() if c["name"] == case)
    inputs = [z[f"{case}/in{i}"] for i in range(c["inputs"])]
    ref = z[f"{case}/out"]
    got, flag = _oracle_run(oracle, c["op"], inputs, c["kwargs"])
    if c["flag"] is not None:
        assert bool(flag) == bool(c["flag"]), case
    if c["op"] == "softmax" and c["flag"]:
        return  # a row with no finite entry: the call fails; its values are not part of the contract
    if c["op"] in REF_BITEXACT:
        if got.dtype == np.float32:
            # bit for bit, except that any NaN matches any NaN (the GPU returns its canonical
            # NaN where x86 propagates a payload)
            both_nan = np.isnan(got) & np.isnan(ref)
            np.testing.assert_array_equal(np.where(both_nan, 0, got.view(np.uint32)),
                                          np.where(both_nan, 0, ref.view(np.uint32)), err_msg=case)
        else:
            np.testing.assert_array_equal(got, ref, err_msg=case)
        return
    ok = np.isfinite(ref)
    np.testing.assert_array_equal(np.isfinite(got), ok, err_msg=case)
    g, r = got[ok].astype(np.float64), ref[ok].astype(np.float64)
    err = float(np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-30))
    assert err <= REF_TOL.get(c["op"], 1e-6), (case, err)
