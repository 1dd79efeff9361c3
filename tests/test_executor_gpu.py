"""GPU: the executor's ProviderExecutionApi behaviour (src/executor.rs) and the decoder-layer
chain against the oracle."""
import importlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

KI = None


def inv(*args, **kw):
    mpc = importlib.import_module("magnetar-provider-cuda_b200")
    return mpc.KernelInvocation(*args, **kw)


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_write_read_and_release(executor):
    x = np.arange(12, dtype=np.float32).reshape(4, 3)
    executor.write_tensor("x", x)
    np.testing.assert_array_equal(executor.read_tensor("x"), x)
    np.testing.assert_array_equal(executor.read_tensor_rows("x", 3, 1), x[3:])
    np.testing.assert_array_equal(executor.read_tensor_rows("x", 1, 2), x[1:3])
    assert executor.read_tensor_rows("x", 3, 2) is None
    assert executor.resident_shape("x") == (4, 3)
    assert executor.release_tensor("x") and not executor.release_tensor("x")
    assert executor.read_tensor("x") is None


def test_zeroed_tensor_needs_no_upload(executor):
    before = executor.kernels.upload_count()
    executor.write_zeroed_tensor("z", (5, 3))
    assert executor.kernels.upload_count() == before
    np.testing.assert_array_equal(executor.read_tensor("z"), np.zeros((5, 3), np.float32))


def test_back_to_back_kernels_do_not_round_trip_through_host(executor, oracle):
    # src/tests_conformance.rs:970-1004
    a = np.array([[1, 2], [3, 4]], np.float32)
    b = np.array([[5, 6], [7, 8]], np.float32)
    executor.write_tensor("a", a)
    executor.write_tensor("b", b)
    k = executor.kernels
    up, down = k.upload_count(), k.download_count()
    executor.run(inv("add", ["a", "b"], "sum"))
    executor.run(inv("mul", ["sum", "b"], "prod"))
    assert k.upload_count() == up and k.download_count() == down
    np.testing.assert_array_equal(executor.read_tensor("prod"), (a + b) * b)
    assert k.download_count() == down + 1


def test_dispatch_errors_are_categorised(executor):
    executor.write_tensor("a", np.ones((2, 2), np.float32))
    r = executor.submit_kernel(inv("no-such-kernel", ["a"], "o"))
    assert not r.success and r.error_code == "KernelNotFound"
    r = executor.submit_kernel(inv("add", ["a", "missing"], "o"))
    assert not r.success and r.error_code == "ExecutionFailed"
    r = executor.submit_kernel(inv("add", ["a", "a"], "o", deadline_millis=0))
    assert not r.success and r.error_code == "KernelTimeout"
    r = executor.submit_kernel(inv("rope", ["a"], "o"))  # no dimension
    assert not r.success and r.error_code == "KernelAttributeUnsupported"
    r = executor.submit_kernel(inv("rope", ["a"], "o", {"dimension": 2, "rotation_pairing": "neox"}))
    assert not r.success and r.error_code == "KernelAttributeUnsupported"
    r = executor.submit_kernel(inv("matmul", ["a", "a"], "o", {"accumulation_dtype": "bf16"}))
    assert not r.success and r.error_code == "DTypeUnsupported"
    r = executor.submit_kernel(inv("rmsnorm", ["a"], "o", {"with_scale": True}))
    assert not r.success and r.error_code == "KernelAttributeUnsupported"
    obs = executor.observations()
    assert obs["failed"] >= 7


def test_failed_dispatch_keeps_previous_output(executor):
    executor.write_tensor("t", np.ones((4, 2), np.float32))
    executor.write_tensor("ids", np.array([0, 1], np.float32))
    executor.run(inv("embedding", ["t", "ids"], "e"))
    prev = executor.read_tensor("e")
    executor.write_tensor("bad", np.array([0, 9], np.float32))
    r = executor.submit_kernel(inv("embedding", ["t", "bad"], "e"))
    assert not r.success and r.error_code == "ShapeUnsupported"
    np.testing.assert_array_equal(executor.read_tensor("e"), prev)


def test_output_buffer_is_reused(executor):
    executor.write_tensor("a", np.ones((64, 64), np.float32))
    executor.run(inv("add", ["a", "a"], "o"))
    p1 = executor.buffer("o").data_ptr()
    executor.run(inv("mul", ["a", "a"], "o"))
    assert executor.buffer("o").data_ptr() == p1
    np.testing.assert_array_equal(executor.read_tensor("o"), np.ones((64, 64), np.float32))


def test_half_ops_through_the_executor(executor, oracle):
    a = np.array([1.0, 2.5, 3.0, -4.25, 0.1, 100.0], np.float32)
    b = np.array([6.0, 0.2, 4.0, 3.0, 0.2, -99.5], np.float32)
    executor.write_tensor("a", a)
    executor.write_tensor("b", b)
    for dtype in ("f16", "bf16"):
        for op in ("add", "mul"):
            executor.run(inv(f"{op}-half", ["a", "b"], "o", input_dtypes=[dtype, dtype]))
            exp = oracle.half_binary_f32(a, b, dtype, op)
            np.testing.assert_array_equal(executor.read_tensor("o").view(np.uint32), exp.view(np.uint32))
    r = executor.submit_kernel(inv("add-half", ["a", "b"], "o"))
    assert not r.success and r.error_code == "DTypeUnsupported"


def test_attribute_defaults_follow_the_reference(executor, oracle):
    r = np.random.default_rng(0)
    x = r.standard_normal((16, 32)).astype(np.float32)
    w = r.standard_normal(32).astype(np.float32)
    executor.write_tensor("x", x)
    executor.write_tensor("w", w)
    executor.run(inv("rmsnorm", ["x", "w"], "n"))  # epsilon defaults to 1e-6
    assert rel(executor.read_tensor("n"), oracle.rmsnorm(x, w, 1e-6)) < 1e-5
    executor.run(inv("rope", ["x"], "r", {"dimension": 8, "head_count": 4}))  # base 10000, interleaved
    assert rel(executor.read_tensor("r"), oracle.rope(x, dimension=8, head_count=4)) < 1e-5
    executor.run(inv("attention", ["x", "x", "x"], "at", {"head_count": 4, "head_dimension": 8}))  # not causal
    assert rel(executor.read_tensor("at"), oracle.attention(x, x, x, 4, 8)) < 1e-4
    executor.run(inv("activation", ["x"], "s", {"kind": "scale", "factor": 0.25}))
    np.testing.assert_array_equal(executor.read_tensor("s"), x * np.float32(0.25))


def _oracle_layer(orc, cfg, w):
    x, bad = orc.embedding(w["table"], w["ids"])
    assert not bad
    h = orc.rmsnorm(x, w["attn_norm"], cfg.eps)
    q, k, v = (orc.matmul(h, w[n]) for n in ("wq", "wk", "wv"))
    q = orc.rope(q, base=cfg.rope_theta, dimension=cfg.head_dim, head_count=cfg.heads)
    k = orc.rope(k, base=cfg.rope_theta, dimension=cfg.head_dim, head_count=cfg.heads)
    a = orc.attention(q, k, v, cfg.heads, cfg.head_dim, causal=True)
    x2 = orc.matmul(a, w["wo"], addend=x, addend_mode=2)
    h2 = orc.rmsnorm(x2, w["mlp_norm"], cfg.eps)
    g = orc.gated_matmul(h2, w["wg"], w["wu"])
    return orc.matmul(g, w["wd"], addend=x2, addend_mode=2)


def test_decoder_layer_matches_oracle_and_capture_replays(executor, oracle):
    layer = importlib.import_module("magnetar-provider-cuda_b200.layer")
    cfg = layer.DecoderLayerConfig()
    w = layer.make_inputs(cfg, seed=0)
    layer.load(executor, w)
    layer.forward(executor, cfg)
    got = executor.read_tensor("out")
    exp = _oracle_layer(oracle, cfg, w)
    assert rel(got, exp) <= 1e-4
    # step capture: the replayed graph produces the same values
    layer.capture(executor, cfg)
    executor.write_zeroed_tensor("scratch", (1,))
    executor.replay_steps(3)
    # The capture launches q, k and v as one grouped projection, whose split-k sums associate
    # differently from three separate launches: equal up to f32 rounding.
    assert rel(executor.read_tensor("out"), got) <= 1e-6
    # a new id vector written into the same buffer flows through the replay
    ids2 = np.random.default_rng(1).integers(0, cfg.vocab, cfg.seq).astype(np.float32)
    buf = executor.buffer("ids")
    from importlib import import_module
    executor.kernels  # same device
    import ctypes
    native = import_module("magnetar-provider-cuda_b200._native")
    native.check(native.lib().mg_buffer_upload(buf.handle, ids2.ctypes.data, ids2.nbytes))
    executor.replay_step()
    w2 = dict(w, ids=ids2)
    assert rel(executor.read_tensor("out"), _oracle_layer(oracle, cfg, w2)) <= 1e-4
    # an invalid id is reported after the replay
    bad = ids2.copy()
    bad[5] = cfg.vocab + 3
    native.check(native.lib().mg_buffer_upload(buf.handle, bad.ctypes.data, bad.nbytes))
    from importlib import import_module as im
    mpc = im("magnetar-provider-cuda_b200")
    with pytest.raises(mpc.CudaError) as e:
        executor.replay_step()
    assert e.value.code == "ShapeUnsupported"


def test_softmax_cannot_be_captured(executor):
    executor.write_tensor("x", np.ones((2, 4), np.float32))
    executor.run(inv("softmax", ["x"], "s"))
    executor.begin_step_capture()
    r = executor.submit_kernel(inv("softmax", ["x"], "s"))
    executor.abort_step_capture()
    assert not r.success and r.error_code == "CaptureUnsupported"


def _zero(executor, ids):
    native = importlib.import_module("magnetar-provider-cuda_b200._native")
    for n in ids:
        b = executor.buffer(n)
        z = np.zeros(b.shape, np.float32)
        native.check(native.lib().mg_buffer_upload(b.handle, z.ctypes.data, z.nbytes))


def test_capture_fuses_projections_of_one_input_and_their_ropes(executor, oracle):
    # q, k, v = h W_q, h W_k, h W_v and rope(q), rope(k): captured, one grouped launch with the
    # rotation in its epilogue; every output id still holds its value after a replay.
    r = np.random.default_rng(3)
    m, d, heads = 128, 256, 4
    h = r.standard_normal((m, d)).astype(np.float32)
    ws = {n: (r.standard_normal((d, d)) * 0.05).astype(np.float32) for n in ("wq", "wk", "wv")}
    executor.write_tensor("h", h)
    for n, w in ws.items():
        executor.write_weight_tensor(n, w)
    attrs = {"dimension": 64, "head_count": heads, "base": 10000.0, "position_offset": 3}
    invs = [inv("matmul", ["h", "wq"], "q"), inv("matmul", ["h", "wk"], "k"), inv("matmul", ["h", "wv"], "v"),
            inv("rope", ["q"], "qr", attrs), inv("rope", ["k"], "kr", attrs)]
    for i in invs:
        executor.run(i)
    names = ("q", "k", "v", "qr", "kr")
    eager = {n: executor.read_tensor(n) for n in names}
    executor.begin_step_capture()
    for i in invs:
        executor.run(i)
    executor.end_step_capture()
    _zero(executor, names)
    before = executor.kernels.launch_count()
    executor.replay_steps(1)
    assert executor.kernels.launch_count() - before == 1  # one grouped launch
    q = oracle.matmul(h, ws["wq"])
    k = oracle.matmul(h, ws["wk"])
    exp = {"q": q, "k": k, "v": oracle.matmul(h, ws["wv"]),
           "qr": oracle.rope(q, base=10000.0, dimension=64, head_count=heads, position_offset=3),
           "kr": oracle.rope(k, base=10000.0, dimension=64, head_count=heads, position_offset=3)}
    for n in names:
        got = executor.read_tensor(n)
        assert rel(got, eager[n]) <= 1e-6, n
        assert rel(got, exp[n]) <= 1e-4, n


def test_capture_does_not_fuse_what_it_must_not(executor, oracle):
    # A chained matmul (reads a deferred output), a half-split rope, a projection of another
    # width and a lone matmul: each launches on its own, with the eager results.
    r = np.random.default_rng(4)
    h = r.standard_normal((128, 128)).astype(np.float32)
    w1 = (r.standard_normal((128, 128)) * 0.1).astype(np.float32)
    w2 = (r.standard_normal((128, 64)) * 0.1).astype(np.float32)
    w3 = (r.standard_normal((128, 128)) * 0.1).astype(np.float32)
    executor.write_tensor("h", h)
    for n, w in (("w1", w1), ("w2", w2), ("w3", w3)):
        executor.write_weight_tensor(n, w)
    half = {"dimension": 64, "head_count": 2, "rotation_pairing": "half_split"}
    invs = [inv("matmul", ["h", "w1"], "a"), inv("matmul", ["a", "w3"], "b"),   # chain
            inv("matmul", ["h", "w2"], "c"), inv("rope", ["b"], "br", half),   # other width, half-split
            inv("matmul", ["b", "w2"], "e")]
    for i in invs:
        executor.run(i)
    names = ("a", "b", "c", "br", "e")
    eager = {n: executor.read_tensor(n) for n in names}
    executor.begin_step_capture()
    for i in invs:
        executor.run(i)
    executor.end_step_capture()
    _zero(executor, names)
    executor.replay_steps(1)
    for n in names:  # nothing was grouped: bit-identical to the eager launches
        np.testing.assert_array_equal(executor.read_tensor(n), eager[n], err_msg=n)


@pytest.mark.parametrize("scaled", [False, True])
def test_capture_fuses_an_embedding_and_the_rmsnorm_of_its_rows(executor, oracle, scaled):
    # embedding -> x, rmsnorm(x, gain) -> h: captured, one launch writing both, each equal bit
    # for bit to the two separate launches; an invalid id is still reported after the replay.
    mpc = importlib.import_module("magnetar-provider-cuda_b200")
    native = importlib.import_module("magnetar-provider-cuda_b200._native")
    r = np.random.default_rng(5)
    vocab, dim, n = 1000, 512, 96
    table = r.standard_normal((vocab, dim)).astype(np.float32)
    gain = (1.0 + 0.1 * r.standard_normal(dim)).astype(np.float32)
    ids = r.integers(0, vocab, n).astype(np.float32)
    executor.write_weight_tensor("table", table)
    executor.write_weight_tensor("gain", gain)
    executor.write_tensor("ids", ids)
    attrs = {"scale": 0.5} if scaled else {}
    invs = [inv("embedding", ["table", "ids"], "x", attrs), inv("rmsnorm", ["x", "gain"], "h", {"epsilon": 1e-5})]
    for i in invs:
        executor.run(i)
    eager = {k: executor.read_tensor(k) for k in ("x", "h")}
    x_exp = table[ids.astype(np.int64)] * (0.5 if scaled else 1.0)
    np.testing.assert_array_equal(eager["x"], x_exp)
    assert rel(eager["h"], oracle.rmsnorm(x_exp, gain, 1e-5)) <= 1e-5
    executor.begin_step_capture()
    for i in invs:
        executor.run(i)
    executor.end_step_capture()
    _zero(executor, ("x", "h"))
    before = executor.kernels.launch_count()
    executor.replay_steps(1)
    assert executor.kernels.launch_count() - before == 1  # one fused launch
    for k in ("x", "h"):
        np.testing.assert_array_equal(executor.read_tensor(k), eager[k], err_msg=k)
    bad = ids.copy()
    bad[7] = vocab + 1
    native.check(native.lib().mg_buffer_upload(executor.buffer("ids").handle, bad.ctypes.data, bad.nbytes))
    with pytest.raises(mpc.CudaError) as e:
        executor.replay_step()
    assert e.value.code == "ShapeUnsupported"


def test_capture_keeps_an_embedding_apart_when_it_must(executor, oracle):
    # An rmsnorm of another tensor, an rmsnorm over head slices (its rows are not the
    # embedding's), and an embedding followed by a matmul of its rows: each launches on its
    # own, with the eager results.
    r = np.random.default_rng(6)
    vocab, dim, n = 500, 256, 64
    table = r.standard_normal((vocab, dim)).astype(np.float32)
    gain = (1.0 + 0.1 * r.standard_normal(dim)).astype(np.float32)
    w = (r.standard_normal((dim, dim)) * 0.05).astype(np.float32)
    y = r.standard_normal((n, dim)).astype(np.float32)
    executor.write_weight_tensor("table", table)
    executor.write_weight_tensor("gain", gain)
    executor.write_weight_tensor("w", w)
    executor.write_tensor("ids", r.integers(0, vocab, n).astype(np.float32))
    executor.write_tensor("y", y)
    invs = [inv("embedding", ["table", "ids"], "x"), inv("rmsnorm", ["y", "gain"], "hy", {"epsilon": 1e-5}),
            inv("embedding", ["table", "ids"], "x2"),
            inv("rmsnorm", ["x2"], "hx", {"epsilon": 1e-5, "head_count": 4, "head_dimension": 64}),
            inv("embedding", ["table", "ids"], "x3"), inv("matmul", ["x3", "w"], "m")]
    for i in invs:
        executor.run(i)
    names = ("x", "hy", "x2", "hx", "x3", "m")
    eager = {k: executor.read_tensor(k) for k in names}
    executor.begin_step_capture()
    for i in invs:
        executor.run(i)
    executor.end_step_capture()
    _zero(executor, names)
    before = executor.kernels.launch_count()
    executor.replay_steps(1)
    assert executor.kernels.launch_count() - before == 6
    for k in names:
        np.testing.assert_array_equal(executor.read_tensor(k), eager[k], err_msg=k)


def test_kv_write_in_place_and_into_a_copy(executor):
    # src/executor.rs:1366-1420: output == store writes the store in place; another output
    # id gets a copy of the store with the rows written, the store unchanged.
    r = np.random.default_rng(7)
    cache = r.standard_normal((16, 8)).astype(np.float32)
    new = r.standard_normal((2, 8)).astype(np.float32)
    executor.write_tensor("cache", cache)
    executor.write_tensor("new", new)
    before = executor.buffer("cache").handle.value
    executor.run(inv("kv-write", ["cache", "new"], "cache", {"row_offset": 5}))
    exp = cache.copy()
    exp[5:7] = new
    np.testing.assert_array_equal(executor.read_tensor("cache"), exp)
    assert executor.buffer("cache").handle.value == before  # the same device buffer
    executor.run(inv("kv-write", ["cache", "new"], "copy", {"row_offset": 14}))
    exp2 = exp.copy()
    exp2[14:16] = new
    np.testing.assert_array_equal(executor.read_tensor("copy"), exp2)
    np.testing.assert_array_equal(executor.read_tensor("cache"), exp)
    r1 = executor.submit_kernel(inv("kv-write", ["cache", "new"], "cache"))
    assert not r1.success and r1.error_code == "KernelAttributeUnsupported"
    r2 = executor.submit_kernel(inv("kv-write", ["cache", "new"], "cache", {"row_offset": 15}))
    assert not r2.success and r2.error_code == "ShapeUnsupported"
    np.testing.assert_array_equal(executor.read_tensor("cache"), exp)


def test_captured_decode_step_replays_at_advancing_offsets(executor, oracle):
    # A decode step -- RoPE of the new query and key at the step's position, the new key and
    # value written into the KV history in place, attention of the one query row over the
    # history -- captured once with position_offset, row_offset and key_count advancing
    # (src/kernels.rs:1019-1062, 1343-1349) and replayed at offsets 0, 1, 2, ... with the
    # step's inputs written into the captured buffers each time.
    mpc = importlib.import_module("magnetar-provider-cuda_b200")
    native = importlib.import_module("magnetar-provider-cuda_b200._native")
    r = np.random.default_rng(8)
    cap, prefix, heads, kvh, d = 300, 40, 4, 2, 64
    kc = np.zeros((cap, kvh * d), np.float32)
    vc = np.zeros((cap, kvh * d), np.float32)
    kc[:prefix] = r.standard_normal((prefix, kvh * d))
    vc[:prefix] = r.standard_normal((prefix, kvh * d))
    executor.write_tensor("kc", kc)
    executor.write_tensor("vc", vc)

    def step_inputs(t):
        g = np.random.default_rng(100 + t)
        return (g.standard_normal((1, heads * d)).astype(np.float32),
                g.standard_normal((1, kvh * d)).astype(np.float32),
                g.standard_normal((1, kvh * d)).astype(np.float32))

    q0, k0, v0 = step_inputs(0)
    for n, x in (("q", q0), ("k", k0), ("v", v0)):
        executor.write_tensor(n, x)
    invs = [inv("rope", ["q"], "qr", {"dimension": d, "head_count": heads, "position_offset": prefix}),
            inv("rope", ["k"], "kr", {"dimension": d, "head_count": kvh, "position_offset": prefix}),
            inv("kv-write", ["kc", "kr"], "kc", {"row_offset": prefix}),
            inv("kv-write", ["vc", "v"], "vc", {"row_offset": prefix}),
            inv("attention", ["qr", "kc", "vc"], "o",
                {"head_count": heads, "head_dimension": d, "kv_head_count": kvh, "causal": True,
                 "key_count": prefix + 1})]
    executor.begin_step_capture(advancing=("position_offset", "row_offset", "key_count"))
    for i in invs:
        executor.run(i)
    executor.end_step_capture()
    assert executor.step_max_offset() == cap - prefix - 1
    kc_exp, vc_exp = kc.copy(), vc.copy()
    for t in range(6):
        q, k, v = step_inputs(t)
        for n, x in (("q", q), ("k", k), ("v", v)):
            native.check(native.lib().mg_buffer_upload(executor.buffer(n).handle, x.ctypes.data, x.nbytes))
        executor.replay_step(offset=t)
        pos = prefix + t
        qr = oracle.rope(q, base=10000.0, dimension=d, head_count=heads, position_offset=pos)
        kr = oracle.rope(k, base=10000.0, dimension=d, head_count=kvh, position_offset=pos)
        kc_exp[pos] = kr[0]
        vc_exp[pos] = v[0]
        exp = oracle.attention(qr, kc_exp[:pos + 1], vc_exp[:pos + 1], heads, d, kv_head_count=kvh, causal=True)
        assert rel(executor.read_tensor("o"), exp) <= 1e-4, t
    assert rel(executor.read_tensor("kc"), kc_exp) <= 1e-5
    np.testing.assert_array_equal(executor.read_tensor("vc"), vc_exp)
    with pytest.raises(mpc.CudaError) as e:
        executor.replay_step(offset=cap - prefix)  # would write past the history
    assert e.value.code == "CaptureUnsupported"


def test_layered_forms_through_the_executor(executor, oracle):
    # src/executor.rs:1798-1965: gelu's approximate, activation sigmoid / softcap, row-scale,
    # concat rows / heads and batched-matmul with their attribute rules
    r = np.random.default_rng(9)
    x = r.standard_normal((6, 16)).astype(np.float32)
    s = r.standard_normal((6, 1)).astype(np.float32)
    y = r.standard_normal((6, 8)).astype(np.float32)
    w = r.standard_normal((2 * 8, 3)).astype(np.float32)
    for n, t in (("x", x), ("s", s), ("y", y), ("w", w)):
        executor.write_tensor(n, t)
    executor.run(inv("gelu", ["x"], "g", {"approximate": "tanh"}))
    assert rel(executor.read_tensor("g"), oracle.gelu_tanh(x)) <= 1e-5
    executor.run(inv("gelu", ["x"], "g2"))
    np.testing.assert_array_equal(executor.read_tensor("g2"), executor.read_tensor("g"))
    r1 = executor.submit_kernel(inv("gelu", ["x"], "g3", {"approximate": "none"}))
    assert not r1.success and r1.error_code == "KernelAttributeUnsupported"
    executor.run(inv("activation", ["x"], "sg", {"kind": "sigmoid"}))
    assert rel(executor.read_tensor("sg"), oracle.sigmoid(x)) <= 1e-5
    executor.run(inv("activation", ["x"], "sc", {"kind": "softcap", "cap": 2.0}))
    assert rel(executor.read_tensor("sc"), oracle.softcap(x, 2.0)) <= 1e-5
    r2 = executor.submit_kernel(inv("activation", ["x"], "sc2", {"kind": "softcap"}))
    assert not r2.success and r2.error_code == "KernelAttributeUnsupported"
    executor.run(inv("row-scale", ["x", "s"], "rs"))
    np.testing.assert_array_equal(executor.read_tensor("rs"), oracle.row_scale(x, s.reshape(-1)))
    executor.run(inv("concat", ["x", "x"], "cr"))
    np.testing.assert_array_equal(executor.read_tensor("cr"), np.concatenate([x, x]))
    executor.run(inv("concat", ["x", "y"], "ch", {"axis": "heads", "head_count": 2}))
    np.testing.assert_array_equal(executor.read_tensor("ch"), oracle.concat_heads(x, y, 2))
    r3 = executor.submit_kernel(inv("concat", ["x", "y"], "cb", {"axis": "columns"}))
    assert not r3.success and r3.error_code == "KernelAttributeUnsupported"
    executor.run(inv("batched-matmul", ["x", "w"], "bm", {"group_count": 2}))
    assert rel(executor.read_tensor("bm"), oracle.batched_matmul(x, w, 2)) <= 1e-4
    r4 = executor.submit_kernel(inv("batched-matmul", ["x", "w"], "bm2"))
    assert not r4.success and r4.error_code == "KernelAttributeUnsupported"


def test_select_greedy_column_over_a_resident_tensor(executor, oracle):
    # src/executor.rs:2549-2563: one reduction and an 8-byte read instead of the row
    r = np.random.default_rng(29)
    logits = r.standard_normal((3, 32000)).astype(np.float32)
    executor.write_tensor("logits", logits)
    k = executor.kernels
    down = k.download_count()
    for row in range(3):
        assert executor.select_greedy_column("logits", row) == oracle.greedy_select(logits, row)
    assert k.download_count() == down + 3
    assert executor.select_greedy_column("logits", 1, [(0, 16000)], 0.8) == oracle.greedy_select(logits, 1, [(0, 16000)], 0.8)
    assert executor.select_greedy_column("logits", 3) is None  # a row past the logits
    assert executor.select_greedy_column("missing", 0) is None


def test_packed_weight_through_the_executor(executor, oracle):
    # src/executor.rs:404-420: write_packed_weight_tensor, then matmul / gated-matmul invocations
    # read it packed; a captured decode step over packed weights replays to the same result
    from q8_cases import activations, packed_q8
    k, n = 128, 64
    gate, up = packed_q8(n, k, 21), packed_q8(n, k, 22)
    executor.write_packed_weight_tensor("gate", gate, n, k)
    executor.write_packed_weight_tensor("up", up, n, k)
    a = activations(1, k, 9)
    executor.write_tensor("x", a)
    executor.run(inv("gated-matmul", ["x", "gate", "up"], "h"))
    expected = oracle.gated_matmul(a, oracle.q8_0_dequantize(gate, n, k), oracle.q8_0_dequantize(up, n, k))
    got = executor.read_tensor("h")
    assert np.all(np.abs(got - expected) <= 1e-5 + 1e-5 * k)
    assert executor.resident_shape("gate") == (k, n)
    np.testing.assert_array_equal(executor.read_tensor("gate"), oracle.q8_0_dequantize(gate, n, k))
    executor.begin_step_capture()
    executor.run(inv("gated-matmul", ["x", "gate", "up"], "h2"))
    executor.end_step_capture()
    executor.replay_step()
    np.testing.assert_array_equal(executor.read_tensor("h2"), got)
    executor.copy_tensor("gate", "gate_copy")
    np.testing.assert_array_equal(executor.read_tensor("gate_copy"), oracle.q8_0_dequantize(gate, n, k))


def test_replay_step_with_host_io(executor, oracle, mpc):
    # replay_step(id, offset, inputs) with the outputs read in the same call: new ids flow in,
    # the layer's output comes back, one synchronisation; a bad id is still reported
    layer = importlib.import_module("magnetar-provider-cuda_b200.layer")
    cfg = layer.DecoderLayerConfig()
    w = layer.make_inputs(cfg, seed=0)
    layer.load(executor, w)
    layer.forward(executor, cfg)
    layer.capture(executor, cfg)
    out = np.empty((cfg.seq, cfg.hidden), np.float32)
    for seed in (1, 2):
        ids = np.random.default_rng(seed).integers(0, cfg.vocab, cfg.seq).astype(np.float32)
        executor.replay_step_io({"ids": ids}, {"out": out})
        assert rel(out, _oracle_layer(oracle, cfg, dict(w, ids=ids))) <= 1e-4
        np.testing.assert_array_equal(out, executor.read_tensor("out"))
    bad = ids.copy()
    bad[0] = -1.0
    with pytest.raises(mpc.CudaError) as e:
        executor.replay_step_io({"ids": bad}, {"out": out})
    assert e.value.code == "ShapeUnsupported"
    with pytest.raises(mpc.CudaError) as e:  # bytes must match the buffer
        executor.replay_step_io({"ids": ids[:5].copy()})
    assert e.value.code == "ShapeUnsupported"
    with pytest.raises(mpc.CudaError) as e:
        executor.replay_step_io(outputs={"missing": out})
    assert e.value.code == "ExecutionFailed"


def test_replay_step_with_pinned_host_io(executor, oracle, mpc):
    # Pinned host buffers take the one-launch form: the step's own nodes with the SMs' copies
    # before its first nodes and after its last kernels (the output copy hangs off them by
    # programmatic edges and waits for them in the kernel).  The output buffer is cleared
    # before each replay so that a copy that ran early would show.
    torch = pytest.importorskip("torch")
    layer = importlib.import_module("magnetar-provider-cuda_b200.layer")
    cfg = layer.DecoderLayerConfig()
    w = layer.make_inputs(cfg, seed=0)
    layer.load(executor, w)
    layer.forward(executor, cfg)
    layer.capture(executor, cfg)
    ids_h = torch.empty(cfg.seq, dtype=torch.float32).pin_memory()
    out_h = torch.empty((cfg.seq, cfg.hidden), dtype=torch.float32).pin_memory()
    replay = executor.step_io({"ids": ids_h}, {"out": out_h})
    for seed in (1, 2, 3):
        ids = np.random.default_rng(seed).integers(0, cfg.vocab, cfg.seq).astype(np.float32)
        ids_h.numpy()[:] = ids
        out_h.fill_(float("nan"))
        replay()
        got = out_h.numpy().copy()
        assert rel(got, _oracle_layer(oracle, cfg, dict(w, ids=ids))) <= 1e-4
        np.testing.assert_array_equal(got, executor.read_tensor("out"))
    ids_h[0] = -1.0  # the embedding-id word rides along with the output copy
    with pytest.raises(mpc.CudaError) as e:
        replay()
    assert e.value.code == "ShapeUnsupported"


def test_pinned_host_io_replays_a_decode_step_at_advancing_offsets(executor, oracle):
    # The advancing form with pinned host I/O: the replay's offset word is a copy node before the
    # step's first nodes, the query, key and value rows come in and the attention output goes
    # out in the same launch, at offsets 0, 1, 2, ...
    torch = pytest.importorskip("torch")
    r = np.random.default_rng(9)
    cap, prefix, heads, kvh, d = 200, 30, 4, 2, 64
    kc = np.zeros((cap, kvh * d), np.float32)
    vc = np.zeros((cap, kvh * d), np.float32)
    kc[:prefix] = r.standard_normal((prefix, kvh * d))
    vc[:prefix] = r.standard_normal((prefix, kvh * d))
    executor.write_tensor("kc", kc)
    executor.write_tensor("vc", vc)
    pinned = {n: torch.zeros((1, w), dtype=torch.float32).pin_memory()
              for n, w in (("q", heads * d), ("k", kvh * d), ("v", kvh * d))}
    for n, x in pinned.items():
        executor.write_tensor(n, x.numpy())
    o_h = torch.empty((1, heads * d), dtype=torch.float32).pin_memory()
    invs = [inv("rope", ["q"], "qr", {"dimension": d, "head_count": heads, "position_offset": prefix}),
            inv("rope", ["k"], "kr", {"dimension": d, "head_count": kvh, "position_offset": prefix}),
            inv("kv-write", ["kc", "kr"], "kc", {"row_offset": prefix}),
            inv("kv-write", ["vc", "v"], "vc", {"row_offset": prefix}),
            inv("attention", ["qr", "kc", "vc"], "o",
                {"head_count": heads, "head_dimension": d, "kv_head_count": kvh, "causal": True,
                 "key_count": prefix + 1})]
    executor.begin_step_capture(advancing=("position_offset", "row_offset", "key_count"))
    for i in invs:
        executor.run(i)
    executor.end_step_capture()
    replay = executor.step_io(pinned, {"o": o_h})
    kc_exp, vc_exp = kc.copy(), vc.copy()
    for t in range(5):
        g = np.random.default_rng(200 + t)
        for n, x in pinned.items():
            x.numpy()[:] = g.standard_normal(x.shape).astype(np.float32)
        o_h.fill_(float("nan"))
        replay(t)
        pos = prefix + t
        q, k, v = (pinned[n].numpy() for n in ("q", "k", "v"))
        qr = oracle.rope(q, base=10000.0, dimension=d, head_count=heads, position_offset=pos)
        kr = oracle.rope(k, base=10000.0, dimension=d, head_count=kvh, position_offset=pos)
        kc_exp[pos] = kr[0]
        vc_exp[pos] = v[0]
        exp = oracle.attention(qr, kc_exp[:pos + 1], vc_exp[:pos + 1], heads, d, kv_head_count=kvh, causal=True)
        assert rel(o_h.numpy(), exp) <= 1e-4, t
    np.testing.assert_array_equal(executor.read_tensor("vc"), vc_exp)


def _grow_scratch_and_allocate(mpc, kernels, oracle):
    """Non-captured work that grows every scratch workspace the layer's step uses (a larger
    matmul's A/B splits, attention partials and splits), then allocations that could land on
    freed memory, filled with garbage."""
    r = np.random.default_rng(11)
    a = r.standard_normal((1024, 1024)).astype(np.float32)
    b = r.standard_normal((1024, 1024)).astype(np.float32)
    da, db = kernels.upload(a), kernels.upload(b)
    kernels.matmul(da, db)  # per-call B split at M = 1024 (scratch slots for A and B)
    q = r.standard_normal((1, 32 * 128)).astype(np.float32)
    kv = r.standard_normal((8192, 8 * 128)).astype(np.float32)
    kernels.attention(kernels.upload(q), kernels.upload(kv), kernels.upload(kv), 32, 128, kv_head_count=8,
                      causal=True)  # decode partials
    s = r.standard_normal((512, 16 * 64)).astype(np.float32)
    kernels.attention(kernels.upload(s), kernels.upload(s), kernels.upload(s), 16, 64, causal=True)
    junk = [kernels.upload(np.full((1 << 20,), np.nan, np.float32)) for _ in range(24)]
    kernels.synchronize()
    return junk


def test_replay_after_scratch_growth_reads_live_memory(executor, oracle, mpc):
    # A captured step keeps addressing the workspaces it was captured with: when later calls
    # grow those workspaces, the old blocks must stay allocated for the step (not freed into
    # the pool, where new allocations would reuse them).
    layer = importlib.import_module("magnetar-provider-cuda_b200.layer")
    cfg = layer.DecoderLayerConfig()
    w = layer.make_inputs(cfg, seed=3)
    layer.load(executor, w)
    layer.capture(executor, cfg)
    executor.replay_steps(1)
    exp = _oracle_layer(oracle, cfg, w)
    assert rel(executor.read_tensor("out"), exp) <= 1e-4
    junk = _grow_scratch_and_allocate(mpc, executor.kernels, oracle)
    for _ in range(3):
        executor.replay_steps(1)
        assert rel(executor.read_tensor("out"), exp) <= 1e-4
    for j in junk:
        j.release()


def test_several_captured_steps_replay_and_release(executor, oracle, mpc):
    # Several StepCaptureIds per executor (src/executor.rs:209-340): each step replays with its
    # own inputs and outputs; a released step is gone; the others still replay.
    layer = importlib.import_module("magnetar-provider-cuda_b200.layer")
    cfg = layer.DecoderLayerConfig()
    w = layer.make_inputs(cfg, seed=4)
    layer.load(executor, w)
    layer.forward(executor, cfg)
    executor.synchronize()
    executor.begin_step_capture()
    layer.forward(executor, cfg)
    whole = executor.end_step_capture_id()  # runs once as it ends
    assert rel(executor.read_tensor("out"), _oracle_layer(oracle, cfg, w)) <= 1e-4
    # a second step: the MLP half alone, on its own input
    executor.write_tensor("x2b", executor.read_tensor("x2"))
    executor.begin_step_capture()
    executor.run(inv("rmsnorm", ["x2b", "mlp_norm"], "h2b", {"epsilon": float(cfg.eps)}))
    executor.run(inv("gated-matmul", ["h2b", "wg", "wu"], "gb"))
    executor.run(inv("matmul-residual", ["gb", "wd", "x2b"], "outb"))
    mlp = executor.end_step_capture_id()
    assert mlp != whole and executor.step_capture_count() == 2
    out = np.empty((cfg.seq, cfg.hidden), np.float32)
    for seed in (5, 6):
        ids = np.random.default_rng(seed).integers(0, cfg.vocab, cfg.seq).astype(np.float32)
        executor.replay_capture(whole, inputs={"ids": ids}, outputs={"out": out})
        assert rel(out, _oracle_layer(oracle, cfg, dict(w, ids=ids))) <= 1e-4
        x2 = np.random.default_rng(seed + 10).standard_normal((cfg.seq, cfg.hidden)).astype(np.float32)
        outb = np.empty_like(out)
        executor.replay_capture(mlp, inputs={"x2b": x2}, outputs={"outb": outb})
        h2 = oracle.rmsnorm(x2, w["mlp_norm"], cfg.eps)
        expb = oracle.matmul(oracle.gated_matmul(h2, w["wg"], w["wu"]), w["wd"], addend=x2, addend_mode=2)
        assert rel(outb, expb) <= 1e-4
    # an input the step never read is refused; so is an embedding id out of range (host check)
    with pytest.raises(mpc.CudaError) as e:
        executor.replay_capture(mlp, inputs={"ids": ids})
    assert e.value.code == "CaptureUnsupported" and "was not read" in e.value.detail
    bad = ids.copy()
    bad[3] = cfg.vocab
    with pytest.raises(mpc.CudaError) as e:
        executor.replay_capture(whole, inputs={"ids": bad})
    assert e.value.code == "ShapeUnsupported"
    executor.release_step_capture(whole)
    assert executor.step_capture_count() == 1
    with pytest.raises(mpc.CudaError) as e:
        executor.replay_capture(whole)
    assert e.value.code == "CaptureUnsupported"
    executor.replay_capture(mlp, inputs={"x2b": x2}, outputs={"outb": outb})
    assert rel(outb, expb) <= 1e-4
    executor.release_step_capture(mlp)
    executor.release_step_capture(mlp)  # unknown ids are not an error
    assert executor.step_capture_count() == 0


def test_replay_refuses_storage_that_changed_since_the_capture(executor, oracle, mpc):
    # src/executor.rs replay_step: a resource rewritten into a new buffer after the capture
    # ("no longer has its captured storage"), and a weight the step reads through its operand
    # form, cannot feed a replay.
    layer = importlib.import_module("magnetar-provider-cuda_b200.layer")
    cfg = layer.DecoderLayerConfig()
    w = layer.make_inputs(cfg, seed=5)
    layer.load(executor, w)
    layer.capture(executor, cfg)
    with pytest.raises(mpc.CudaError) as e:  # a step-I/O write into a weight read as an operand form
        executor.replay_step_io({"wq": w["wq"]})
    assert e.value.code == "CaptureUnsupported" and "operand form" in e.value.detail
    executor.replay_steps(1)
    assert rel(executor.read_tensor("out"), _oracle_layer(oracle, cfg, w)) <= 1e-4
    # the weight written in place: its operand form is rebuilt for eager calls, so the step's is gone
    wq2 = (w["wq"] * 0.5).astype(np.float32)
    mpc_native = importlib.import_module("magnetar-provider-cuda_b200._native")
    mpc_native.check(mpc_native.lib().mg_buffer_upload(executor.buffer("wq").handle, wq2.ctypes.data, wq2.nbytes))
    with pytest.raises(mpc.CudaError) as e:
        executor.replay_steps(1)
    assert e.value.code == "CaptureUnsupported" and "wq" in e.value.detail
    # a rewritten id (a new buffer) invalidates the step
    layer.capture(executor, cfg)
    executor.replay_steps(1)
    executor.write_tensor("ids", w["ids"])
    with pytest.raises(mpc.CudaError) as e:
        executor.replay_steps(1)
    assert e.value.code == "CaptureUnsupported" and "no longer has its captured storage" in e.value.detail
    # capturing again makes a step over the current storage
    layer.capture(executor, cfg)
    executor.replay_steps(1)
    assert rel(executor.read_tensor("out"), _oracle_layer(oracle, cfg, dict(w, wq=wq2))) <= 1e-4


def test_observation_log_records_each_dispatch(executor, mpc):
    # src/executor.rs:1082-1100, 1197-1232: Started, then Completed / Failed / Timeout.
    executor.write_tensor("a", np.ones((2, 2), np.float32))
    executor.run(inv("add", ["a", "a"], "b"))
    r = executor.submit_kernel(inv("no-such-kernel", ["a"], "o"))
    assert not r.success
    r = executor.submit_kernel(inv("add", ["a", "a"], "c", deadline_millis=0))
    assert not r.success and r.error_code == "KernelTimeout"
    log = executor.observation_log()
    assert [o["kind"] for o in log[-6:]] == [
        "KernelDispatchStarted", "KernelDispatchCompleted", "KernelDispatchStarted", "KernelDispatchFailed",
        "KernelDispatchStarted", "KernelTimeout"]
    assert [o["kernel"] for o in log[-6:]] == ["add", "add", "no-such-kernel", "no-such-kernel", "add", "add"]
    assert log[-3]["error"] == "KernelNotFound"
    inv_ids = [o["invocation"] for o in log[-6:]]
    assert inv_ids[0] == inv_ids[1] and inv_ids[2] == inv_ids[3] and inv_ids[4] == inv_ids[5]
    assert inv_ids[0] < inv_ids[2] < inv_ids[4]


def test_observation_log_is_bounded(executor):
    executor.write_tensor("a", np.ones((4,), np.float32))
    for _ in range(2100):
        executor.run(inv("add", ["a", "a"], "b"))
    log = executor.observation_log()
    assert len(log) == 4096
    assert log[-1]["kind"] == "KernelDispatchCompleted"
