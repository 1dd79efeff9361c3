"""GPU parity at the BASELINE configurations' own sizes.

Each test runs the provider's kernel at the full configured size (so it takes the same launch
path, tiling, split and cluster layout as the benchmark) and compares a sample of the output
element by element with the CPU oracle run on the matching slice of the input: rows are
independent in softmax, rmsnorm, rope, silu and matmul, and heads are independent in
attention, so the slice is the same computation.  Where the reference's own kernels have been
compiled (``oracle/_ref``, see ``oracle/ref_kernels.py``), the same slices are also run through
them on the GPU and compared.  Bars: rel-L2 <= 1e-5 (elementwise, norm, rope, softmax),
<= 1e-4 (matmul, attention), bit-exact for add/mul/residual-add and the half ops.
"""
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


def ref_kernels():
    """The reference's kernels, or None when oracle/_ref was not built."""
    from oracle import ref_kernels as rk
    return rk if rk.available() else None


def torch_gen(seed):
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return g


# ---------------------------------------------------------------------------------- configs[2]
def test_attention_configs2_full_size_sampled_heads(kernels, oracle):
    """Causal attention b4 h32 d128 s2048 (batch folded into 128 heads), Q/K after RoPE
    theta 1e4 at positions 0..2047; eight heads spread over the four batches checked."""
    import torch
    S, H, D = 2048, 128, 128
    g = torch_gen(31)
    q = torch.randn(S, H * D, device="cuda", generator=g)
    k = torch.randn(S, H * D, device="cuda", generator=g)
    v = torch.randn(S, H * D, device="cuda", generator=g)
    W = kernels.wrap_tensor
    qr = kernels.rope(W(q), base=10000.0, dimension=D, head_count=H)
    kr = kernels.rope(W(k), base=10000.0, dimension=D, head_count=H)
    out = kernels.download(kernels.attention(qr, kr, W(v), H, D, causal=True))
    qn, kn, vn = kernels.download(qr), kernels.download(kr), v.cpu().numpy()
    heads = [0, 17, 42, 63, 64, 90, 111, 127]
    cols = np.concatenate([np.arange(h * D, (h + 1) * D) for h in heads])
    qs, ks, vs = (np.ascontiguousarray(x[:, cols]) for x in (qn, kn, vn))
    exp = oracle.attention(qs, ks, vs, len(heads), D, causal=True)
    got = out[:, cols]
    for i, h in enumerate(heads):
        sl = slice(i * D, (i + 1) * D)
        assert rel(got[:, sl], exp[:, sl]) <= TOL_MATMUL, h
    rk = ref_kernels()
    if rk is not None:
        ref = rk.attention(qs, ks, vs, len(heads), D, causal=True).cpu().numpy()
        assert rel(got, ref) <= TOL_MATMUL
        assert rel(exp, ref) <= 1e-6  # the oracle against the reference itself


def test_softmax_configs2_full_size_sampled_rows(kernels, oracle):
    """Row softmax on [262144, 2048] logits N(0, 4): every 64th row compared."""
    import torch
    R, C = 262144, 2048
    x = torch.randn(R, C, device="cuda", generator=torch_gen(32)) * 2
    y = torch.empty_like(x)
    kernels.softmax_rows(kernels.wrap_tensor(x), out=kernels.wrap_tensor(y))
    rows = torch.arange(0, R, 64, device="cuda")
    xs = x[rows].cpu().numpy()
    got = y[rows].cpu().numpy()
    exp, bad = oracle.softmax(xs)
    assert not bad
    assert rel(got, exp) <= TOL_ELEMENTWISE
    assert float(np.max(np.abs(got - exp))) <= 1e-6
    rk = ref_kernels()
    if rk is not None:
        ref, _ = rk.softmax(xs)
        assert rel(got, ref.cpu().numpy()) <= TOL_ELEMENTWISE
    del x, y


# ---------------------------------------------------------------------------------- configs[1]
@pytest.mark.parametrize("M", [128, 2048, 8192])
@pytest.mark.parametrize("weight", [True, False])
def test_matmul_configs1_every_m_tile(kernels, oracle, M, weight):
    """C = A B, N = K = 4096, A and B N(0, 1/sqrt(K)); B as a prepared weight and per call.
    Two rows of every 128-row tile (its first and its last) are compared over all N columns,
    which covers every output tile of the launch."""
    import torch
    K = N = 4096
    g = torch_gen(40 + M)
    a = torch.randn(M, K, device="cuda", generator=g) / math.sqrt(K)
    b = torch.randn(K, N, device="cuda", generator=g) / math.sqrt(K)
    db = kernels.wrap_tensor(b)
    if weight:
        db.set_weight()
    c = kernels.download(kernels.matmul(kernels.wrap_tensor(a), db))
    rows = sorted(set([t * 128 for t in range(M // 128)] + [t * 128 + 127 for t in range(M // 128)]))
    an, bn = a[rows].cpu().numpy(), b.cpu().numpy()
    exp = oracle.matmul(an, bn)
    assert rel(c[rows], exp) <= TOL_MATMUL
    for t in range(0, len(rows), 2):  # each tile's pair on its own
        assert rel(c[rows[t:t + 2]], exp[t:t + 2]) <= TOL_MATMUL, rows[t]
    rk = ref_kernels()
    if rk is not None and M == 8192:
        ref = rk.matmul(an, bn).cpu().numpy()
        assert rel(c[rows], ref) <= TOL_MATMUL


@pytest.mark.parametrize("M", [1, 16])
def test_matmul_configs1_few_rows_full(kernels, oracle, M):
    """The few-row path at N = K = 4096, every output compared."""
    r = np.random.default_rng(50 + M)
    K = N = 4096
    a = (r.standard_normal((M, K)) / math.sqrt(K)).astype(np.float32)
    b = (r.standard_normal((K, N)) / math.sqrt(K)).astype(np.float32)
    got = kernels.download(kernels.matmul(kernels.upload(a), kernels.upload(b).set_weight()))
    assert rel(got, oracle.matmul(a, b)) <= TOL_MATMUL


# ---------------------------------------------------------------------------------- configs[3]
def test_memory_bound_configs3_full_size(kernels, oracle):
    """[8192, 4096]: rmsnorm (gain N(1, 0.1), eps 1e-5), rope (32 heads x 128, theta 5e5) and
    silu on 512 sampled rows against the oracle; add / mul / residual-add bit-exact on every
    element."""
    import torch
    R, C = 8192, 4096
    g = torch_gen(60)
    x = torch.randn(R, C, device="cuda", generator=g)
    y = torch.randn(R, C, device="cuda", generator=g)
    gain = 1 + 0.1 * torch.randn(C, device="cuda", generator=g)
    W = kernels.wrap_tensor
    dx, dy = W(x), W(y)
    rows = torch.arange(0, R, 16, device="cuda")
    xs = x[rows].cpu().numpy()
    gn = gain.cpu().numpy()
    rk = ref_kernels()
    cases = [
        ("rmsnorm", kernels.rmsnorm(dx, W(gain), 1e-5), oracle.rmsnorm(xs, gn, 1e-5),
         rk.rmsnorm(xs, gn, 1e-5) if rk else None),
        ("rope", kernels.rope(dx, base=500000.0, dimension=128, head_count=32),
         None, None),
        ("silu", kernels.silu(dx), oracle.silu(xs), rk.silu(xs) if rk else None),
    ]
    for name, out, exp, ref in cases:
        got_all = kernels.download(out)
        got = got_all[rows.cpu().numpy()]
        if name == "rope":  # positions are the row indices: the oracle runs on whole rows with their offsets
            exp = np.concatenate([oracle.rope(xs[i:i + 1], base=500000.0, dimension=128, head_count=32,
                                              position_offset=int(rr)) for i, rr in enumerate(rows.tolist())])
            if rk:
                ref = np.concatenate([rk.rope(xs[i:i + 1], base=500000.0, dimension=128, head_count=32,
                                              position_offset=int(rr)).cpu().numpy()
                                      for i, rr in enumerate(rows.tolist()[:32])])
                assert rel(got[:32], ref) <= TOL_ELEMENTWISE
                ref = None
        assert rel(got, exp) <= TOL_ELEMENTWISE, name
        if ref is not None:
            assert rel(got, ref.cpu().numpy()) <= TOL_ELEMENTWISE, name
    xn, yn = x.cpu().numpy(), y.cpu().numpy()
    np.testing.assert_array_equal(kernels.download(kernels.add(dx, dy)), xn + yn)
    np.testing.assert_array_equal(kernels.download(kernels.mul(dx, dy)), xn * yn)
    np.testing.assert_array_equal(kernels.download(kernels.residual_add(dx, dy)), xn + yn)


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_half_ops_configs3_full_size(kernels, oracle, dt):
    """add-half / mul-half on [8192, 4096] with inputs uniform(-8, 8): every element bit-exact."""
    import torch
    tdt = torch.float16 if dt == "f16" else torch.bfloat16
    g = torch_gen(70)
    a = (torch.rand(8192, 4096, device="cuda", generator=g) * 16 - 8).to(tdt)
    b = (torch.rand(8192, 4096, device="cuda", generator=g) * 16 - 8).to(tdt)
    W = kernels.wrap_tensor
    ab, bb = a.view(torch.int16).cpu().numpy().view(np.uint16), b.view(torch.int16).cpu().numpy().view(np.uint16)
    for op, fn in (("add", kernels.add_half), ("mul", kernels.mul_half)):
        got = kernels.download_raw(fn(W(a), W(b)))
        np.testing.assert_array_equal(got, oracle.half_binary(ab, bb, dt, op), err_msg=f"{op} {dt}")


# ---------------------------------------------------------------------------------- configs[4]
def test_tp_mlp_configs4_reduced_shape_on_one_rank(mpc, kernels, oracle):
    """The tensor-parallel SwiGLU MLP at configs[4]'s proportions reduced eight-fold (tokens
    512, hidden 1024, ffn 3584) on one rank: the whole MLP, and the sum of four ranks' shares
    (gate/up column shares, down row shares) computed one after another on this GPU, against
    the oracle on 64 sampled tokens."""
    tp = __import__("importlib").import_module("magnetar-provider-cuda_b200.tensor_parallel")
    T, Hd, F = 512, 1024, 3584
    r = np.random.default_rng(80)
    x = r.standard_normal((T, Hd)).astype(np.float32)
    wg = (r.standard_normal((Hd, F)) * 0.02).astype(np.float32)
    wu = (r.standard_normal((Hd, F)) * 0.02).astype(np.float32)
    wd = (r.standard_normal((F, Hd)) * 0.02).astype(np.float32)
    rows = np.arange(0, T, 8)
    exp = oracle.matmul(oracle.gated_matmul(x[rows], wg, wu), wd)
    group = tp.TpGroup(kernels, 0, 1, tp.TpGroup.unique_id())
    try:
        dx = kernels.upload(x)
        y = kernels.download(group.mlp(dx, kernels.upload(wg), kernels.upload(wu), kernels.upload(wd), chunks=4))
        assert rel(y[rows], exp) <= TOL_MATMUL
        total = np.zeros((T, Hd), np.float64)
        for member in range(4):
            part = group.mlp(dx, kernels.upload(tp.split_columns(wg, 4, member)),
                             kernels.upload(tp.split_columns(wu, 4, member)),
                             kernels.upload(tp.split_rows(wd, 4, member)), chunks=4)
            total += kernels.download(part)
        assert rel(total[rows], exp) <= TOL_MATMUL
    finally:
        group.close()
